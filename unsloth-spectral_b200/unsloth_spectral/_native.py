"""ctypes binding of ``libspx.so`` (declared in ``include/spx.h``).

Only plain pointers, integers and floats cross this boundary.  Tensors are passed by
``data_ptr()`` and the current CUDA stream by its handle.  Every call checks the
returned status and raises; there is no fallback path: when the library is missing
or the device is not sm_100, operations raise ``SpxUnavailable``.
"""
from __future__ import annotations

import ctypes as C
import os

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libspx.so")

SPX_OK = 0
SPX_ERR_WORKSPACE = 5
SPX_ERR_EMPTY = 6
NOALLOC_SCRATCH_BYTES = 64 << 20
SPX_F32, SPX_F16, SPX_BF16 = 0, 1, 2
SPX_ROPE_DISTANCE, SPX_ROPE_ABSOLUTE = 0, 1
SPX_PATH_GENERIC, SPX_PATH_RECONSTRUCT, SPX_PATH_PROJECTION = 0, 1, 2

_DTYPES = {torch.float32: SPX_F32, torch.float16: SPX_F16, torch.bfloat16: SPX_BF16}


class SpxUnavailable(RuntimeError):
    """The CUDA library could not be loaded or the device is unsupported."""


class SpxError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"spx status {status}: {msg}")
        self.status = status


class DecodeArgs(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "num_layers", "batch", "num_q_heads", "num_kv_heads", "head_dim", "block_size", "num_blocks",
        "block_capacity", "rank_k", "rank_v", "hot_len", "hot_capacity", "dtype", "rope_mode", "rope_tied",
        "rope_len")] + [
        ("query_position", C.c_int64), ("scale", C.c_float), ("mask_stride", C.c_int32)] + [
        (n, C.c_void_p) for n in (
            "q", "codes_k", "codes_v", "scale_k", "scale_v", "basis_k", "basis_v", "block_pos", "hot_k",
            "hot_v", "hot_pos", "cos_table", "sin_table", "mask", "out", "workspace")] + [
        ("workspace_bytes", C.c_size_t), ("rope_freq", C.c_void_p), ("hot_len_device", C.c_void_p)]


class RsvdArgs(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("num_mats", "m", "n", "k", "r", "n_iter", "in_dtype")] + [
        ("M", C.c_void_p), ("omega", C.c_void_p), ("U", C.c_void_p), ("S", C.c_void_p), ("Vh", C.c_void_p),
        ("M_mat_stride", C.c_int64), ("codes", C.c_void_p), ("codes_mat_stride", C.c_int64), ("codes_t_stride", C.c_int64),
        ("codes_j_stride", C.c_int64), ("codes_rank_pad", C.c_int32), ("codes_tiled", C.c_int32),
        ("qscale", C.c_void_p),
        ("scale_mat_stride", C.c_int64), ("qminmax", C.c_void_p), ("minmax_mat_stride", C.c_int64),
        ("basis", C.c_void_p), ("basis_dtype", C.c_int32), ("basis_mat_stride", C.c_int64),
        ("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t)]


class QuantArgs(C.Structure):
    _fields_ = [("num_groups", C.c_int32), ("group_elems", C.c_int64), ("x", C.c_void_p),
                ("codes", C.c_void_p), ("scale", C.c_void_p), ("minmax", C.c_void_p), ("dequant", C.c_void_p)]


class ReconstructArgs(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "batch", "num_kv_heads", "head_dim", "block_size", "num_blocks", "block_capacity", "rank",
        "rank_major", "dtype", "out_tokens")] + [
        ("codes", C.c_void_p), ("scale", C.c_void_p), ("basis", C.c_void_p), ("out", C.c_void_p)]


class BlockScoreArgs(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "batch", "num_q_heads", "num_kv_heads", "head_dim", "block_size", "rank", "rope_len")] + [
        ("start_position", C.c_int64)] + [(n, C.c_void_p) for n in (
            "q", "coeffs", "basis", "cos_table", "sin_table", "scores")]


class BlockValueArgs(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "batch", "num_q_heads", "num_kv_heads", "head_dim", "block_size", "rank")] + [
        (n, C.c_void_p) for n in ("attn", "coeffs", "basis", "out")]


class PrefillArgs(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "batch", "num_q_heads", "num_kv_heads", "head_dim", "q_len", "block_size", "num_blocks", "block_capacity",
        "rank_k", "rank_v", "hot_len", "hot_capacity", "dtype", "rope_len", "causal", "mask_dtype")] + [
        ("scale", C.c_float)] + [(n, C.c_void_p) for n in (
            "q", "q_pos", "codes_k", "codes_v", "scale_k", "scale_v", "basis_k", "basis_v", "block_pos", "hot_k",
            "hot_v", "hot_pos", "cos_table", "sin_table", "mask")] + [
        (n, C.c_int64) for n in ("mask_stride_b", "mask_stride_h", "mask_stride_q")] + [("out", C.c_void_p)]


EXPORTS = {
    "spx_decode_workspace_size": (C.c_size_t, [C.POINTER(DecodeArgs)]),
    "spx_decode_attn": (C.c_int, [C.POINTER(DecodeArgs), C.c_void_p]),
    "spx_decode_attn_noalloc": (C.c_int, [C.POINTER(DecodeArgs), C.c_void_p]),
    "spx_decode_path": (C.c_int, [C.POINTER(DecodeArgs)]),
    "spx_rsvd_workspace_size": (C.c_size_t, [C.POINTER(RsvdArgs)]),
    "spx_rsvd_compress": (C.c_int, [C.POINTER(RsvdArgs), C.c_void_p]),
    "spx_quantize_int8": (C.c_int, [C.POINTER(QuantArgs), C.c_void_p]),
    "spx_rope_rows": (C.c_int, [C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int64,
                                C.c_int64, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p]),
    "spx_hot_append": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_void_p,
                                 C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                                 C.c_int, C.c_void_p]),
    "spx_rmsnorm": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int,
                              C.c_float, C.c_int, C.c_void_p]),
    "spx_reconstruct": (C.c_int, [C.POINTER(ReconstructArgs), C.c_void_p]),
    "spx_block_scores": (C.c_int, [C.POINTER(BlockScoreArgs), C.c_void_p]),
    "spx_block_values": (C.c_int, [C.POINTER(BlockValueArgs), C.c_void_p]),
    "spx_prefill_attn": (C.c_int, [C.POINTER(PrefillArgs), C.c_void_p]),
    "spx_abi_version": (C.c_int, []),
    "spx_status_string": (C.c_char_p, [C.c_int]),
    "spx_last_error": (C.c_char_p, []),
    "spx_check_device": (C.c_int, []),
}

ABI_VERSION = 4
_lib = None
_load_error = None
_device_ok = {}


def load(path: str = LIB_PATH):
    """Load (once) and return the ctypes library; raises SpxUnavailable."""
    global _lib, _load_error
    if _lib is not None:
        return _lib
    if _load_error is not None:
        raise SpxUnavailable(_load_error)
    if not os.path.exists(path):
        _load_error = (f"{path} is missing; build it with "
                       f"`python unsloth-spectral_b200/csrc/build.py`")
        raise SpxUnavailable(_load_error)
    try:
        lib = C.CDLL(path)
    except OSError as e:
        _load_error = f"cannot load {path}: {e}"
        raise SpxUnavailable(_load_error) from e
    for name, (res, args) in EXPORTS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.spx_abi_version() != ABI_VERSION:
        _load_error = f"ABI version {lib.spx_abi_version()} != {ABI_VERSION}"
        raise SpxUnavailable(_load_error)
    _lib = lib
    return lib


def available() -> bool:
    try:
        load()
        return True
    except SpxUnavailable:
        return False


def lib_for(device: torch.device):
    """The library, after checking that ``device`` is a CUDA sm_100 device."""
    lib = load()
    if device.type != "cuda":
        raise SpxUnavailable(f"spx kernels run on CUDA sm_100 devices only, got {device}")
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _device_ok:
        with torch.cuda.device(idx):
            _device_ok[idx] = lib.spx_check_device()
    if _device_ok[idx] != SPX_OK:
        raise SpxUnavailable(lib.spx_last_error().decode() or "unsupported device")
    return lib


def check(lib, status: int, what: str):
    if status != SPX_OK:
        msg = lib.spx_last_error().decode() or lib.spx_status_string(status).decode()
        if status == SPX_ERR_EMPTY:
            raise ValueError("Empty cache - no keys available")
        raise SpxError(status, f"{what}: {msg}")


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPES[dt]
    except KeyError:
        raise TypeError(f"unsupported dtype {dt}; expected float32, float16 or bfloat16") from None


def ptr(t) -> int:
    return 0 if t is None else t.data_ptr()


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


_workspaces = {}


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """A cached uint8 scratch buffer of at least ``nbytes`` for ``device`` and its current
    stream (grown on demand and owned by this process; the library never allocates).
    Calls on one stream run in order, so reusing the buffer per stream is race-free."""
    key = (device.type, device.index, torch.cuda.current_stream(device).cuda_stream)
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _workspaces[key] = buf
    return buf
