"""ctypes binding of libmm4.so (the C ABI declared in include/mm4.h).

The library is the only compute path: if it is missing or the device is not
an sm_100 part, calls raise MM4Error — there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libmm4.so")

MM4_OK = 0
MM4_ERR_INVALID = 1
MM4_ERR_UNSUPPORTED = 2
MM4_ERR_CUDA = 3
MM4_ERR_NCCL = 4
MM4_ERR_TIMEOUT = 5
MM4_ERR_WORKSPACE = 6

MM4_ATTN_BHSD = 0
MM4_ATTN_BSHD = 1

WEIGHTS_HWIO, WEIGHTS_OHWI, WEIGHTS_OIHW, WEIGHTS_DHWIO, WEIGHTS_ODHWI, WEIGHTS_OIDHW = range(6)


class MM4Error(RuntimeError):
    """A non-zero mm4_status, with the library's message."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{status_name(status)}: {message}")
        self.status = status


class GemmDesc(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "M", "N", "K", "transpose_left", "transpose_right", "bias", "split_k",
        "block_m", "block_n", "block_k", "cooperative_simdgroups", "preemptive_simdgroups", "swap_mn")]


class AttentionDesc(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int32), ("heads_q", ctypes.c_int32), ("heads_kv", ctypes.c_int32),
                ("rows", ctypes.c_int32), ("columns", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("scale", ctypes.c_float), ("layout", ctypes.c_int32)]


class Conv2dDesc(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "batch_size", "input_height", "input_width", "input_channels", "output_channels",
        "kernel_height", "kernel_width", "stride_y", "stride_x", "dilation_y", "dilation_x",
        "padding_top", "padding_bottom", "padding_left", "padding_right", "weight_layout", "bias")]


class Conv3dDesc(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "batch_size", "input_depth", "input_height", "input_width", "input_channels", "output_channels",
        "kernel_depth", "kernel_height", "kernel_width", "stride_z", "stride_y", "stride_x",
        "dilation_z", "dilation_y", "dilation_x", "padding_top", "padding_bottom", "padding_left",
        "padding_right", "padding_front", "padding_back", "weight_layout", "bias")]


class PeerHandle(ctypes.Structure):
    """mm4_peer_handle: a CUDA IPC memory handle as plain bytes."""
    _fields_ = [("bytes", ctypes.c_ubyte * 64)]


_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_sz = ctypes.c_size_t

# name -> (restype, argtypes); every symbol include/mm4.h declares.
SIGNATURES = {
    "mm4_version": (ctypes.c_int, []),
    "mm4_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "mm4_last_error": (ctypes.c_char_p, []),
    "mm4_device_supported": (ctypes.c_int, []),
    "mm4_check": (ctypes.c_int, [_vp]),
    "mm4_set_wait_timeout_ns": (None, [ctypes.c_uint64]),
    "mm4_get_wait_timeout_ns": (ctypes.c_uint64, []),
    "mm4_debug_wait_timeout": (ctypes.c_int, [ctypes.c_uint64, _vp]),
    "mm4_debug_ex2": (ctypes.c_int, [_vp, _vp, ctypes.c_int64, ctypes.c_int, _vp]),
    "mm4_workspace_clear": (ctypes.c_int, [_vp, _sz, _vp]),
    "mm4_gemm_plan_create": (ctypes.c_int, [ctypes.POINTER(_vp), ctypes.POINTER(GemmDesc)]),
    "mm4_gemm_plan_destroy": (None, [_vp]),
    "mm4_gemm_workspace_size": (_sz, [_vp]),
    "mm4_gemm_plan_kernel_name": (ctypes.c_char_p, [_vp]),
    "mm4_gemm_run": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp, ctypes.c_int]),
    "mm4_gemm_partial_run": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "mm4_splitk_finalize": (ctypes.c_int, [_i32, _i32, _vp, _vp, _vp, _vp]),
    "mm4_gemm_splitk_run_noalloc": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp]),
    "mm4_debug_noalloc_wait_timeout": (ctypes.c_int, [ctypes.c_uint64, _vp]),
    "mm4_peer_alloc": (ctypes.c_int, [_sz, ctypes.POINTER(_vp), ctypes.POINTER(PeerHandle)]),
    "mm4_peer_free": (ctypes.c_int, [_vp]),
    "mm4_peer_open": (ctypes.c_int, [ctypes.POINTER(PeerHandle), ctypes.POINTER(_vp)]),
    "mm4_peer_close": (ctypes.c_int, [_vp]),
    "mm4_splitk_group_exchange_bytes": (ctypes.c_int, [_vp, _i32, ctypes.POINTER(_sz)]),
    "mm4_splitk_group_create": (ctypes.c_int, [ctypes.POINTER(_vp), _vp, _i32, _i32, _i32, ctypes.POINTER(_vp),
                                               _vp]),
    "mm4_splitk_group_destroy": (None, [_vp]),
    "mm4_gemm_splitk_group_run": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp]),
    "mm4_comm_unique_id": (ctypes.c_int, [_vp]),
    "mm4_comm_init": (ctypes.c_int, [ctypes.POINTER(_vp), _i32, _i32, _vp]),
    "mm4_comm_destroy": (None, [_vp]),
    "mm4_gemm_splitk_run_distributed": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, ctypes.c_int]),
    "mm4_attention_plan_create": (ctypes.c_int, [ctypes.POINTER(_vp), ctypes.POINTER(AttentionDesc)]),
    "mm4_attention_plan_destroy": (None, [_vp]),
    "mm4_attention_plan_kernel_name": (ctypes.c_char_p, [_vp]),
    "mm4_attention_fwd": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, ctypes.c_int]),
    "mm4_attention_fwd_lse": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "mm4_conv_run_host": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, ctypes.c_int32, _vp]),
    "mm4_gemm_run_host": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, ctypes.c_int32, _vp]),
    "mm4_attention_fwd_host": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, ctypes.c_int32, _vp]),
    "mm4_attention_bwd_host": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, ctypes.c_size_t, ctypes.c_int32, _vp]),
    "mm4_attention_bwd_workspace_size": (_sz, [_vp]),
    "mm4_attention_bwd": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "mm4_conv2d_plan_create": (ctypes.c_int, [ctypes.POINTER(_vp), ctypes.POINTER(Conv2dDesc)]),
    "mm4_conv3d_plan_create": (ctypes.c_int, [ctypes.POINTER(_vp), ctypes.POINTER(Conv3dDesc)]),
    "mm4_conv_plan_destroy": (None, [_vp]),
    "mm4_conv_plan_kernel_name": (ctypes.c_char_p, [_vp]),
    "mm4_conv_plan_tile_grid": (ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_int32)]),
    "mm4_conv_output_elements": (ctypes.c_int64, [_vp]),
    "mm4_conv_run": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, ctypes.c_int]),
    "mm4_permute_weights": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.POINTER(_i32), _vp, _vp, _vp]),
}

_lib = None
_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    """Loads libmm4.so once; raises MM4Error if it has not been built."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise MM4Error(MM4_ERR_UNSUPPORTED,
                               f"{LIB_PATH} is missing: build it with `python -m example_matmul_metal4_b200.build`")
            handle = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def status_name(status: int) -> str:
    names = {0: "MM4_OK", 1: "MM4_ERR_INVALID", 2: "MM4_ERR_UNSUPPORTED", 3: "MM4_ERR_CUDA", 4: "MM4_ERR_NCCL",
             5: "MM4_ERR_TIMEOUT", 6: "MM4_ERR_WORKSPACE"}
    return names.get(status, f"MM4_ERR_{status}")


def check(status: int) -> None:
    if status != MM4_OK:
        msg = lib().mm4_last_error()
        raise MM4Error(status, msg.decode() if msg else "")


def stream_handle(stream=None) -> int | None:
    """cudaStream_t of a torch stream (default: torch's current stream on the current device). The default
    is read through torch's raw-stream query, which skips building a Stream object (~0.3 us against ~3 us
    per call)."""
    import torch
    if stream is None:
        raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
        if raw is not None:
            return raw(torch._C._cuda_getDevice()) or None
        stream = torch.cuda.current_stream()
    return stream.cuda_stream or None


def sync_check(stream=None) -> None:
    """Synchronises the stream and raises MM4Error if a kernel recorded an error."""
    check(lib().mm4_check(stream_handle(stream)))
