"""ctypes binding of libddtree_b200.so (include/ddtree_b200.h).

This is the only place Python touches the native library.  There is no
fallback: if the library is missing or a CUDA device is required and absent,
the calls raise.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libddtree_b200.so"

DDT_F32, DDT_BF16, DDT_F16, DDT_BOOL = 0, 1, 2, 3
DDT_INFO_NONFINITE = 1

_c_i64 = ctypes.c_int64
_c_p = ctypes.c_void_p


class TreeOutputs(ctypes.Structure):
    _fields_ = [
        ("top_ids", _c_p),
        ("top_lp", _c_p),
        ("node_token_ids", _c_p),
        ("node_depths", _c_p),
        ("parents", _c_p),
        ("visibility", _c_p),
        ("vis_words", _c_i64),
        ("verify_ids", _c_p),
        ("verify_pos", _c_p),
        ("info", _c_p),
    ]


class AttentionArgs(ctypes.Structure):
    _fields_ = [
        ("q", _c_p),
        ("q_stride_tok", _c_i64),
        ("q_stride_head", _c_i64),
        ("k", _c_p),
        ("v", _c_p),
        ("kv_stride_head", _c_i64),
        ("kv_stride_row", _c_i64),
        ("kv_rows", _c_i64),
        ("out", _c_p),
        ("o_stride_tok", _c_i64),
        ("o_stride_head", _c_i64),
        ("n_tokens", _c_i64),
        ("hq", _c_i64),
        ("hkv", _c_i64),
        ("head_dim", _c_i64),
        ("past_length", _c_i64),
        ("visibility", _c_p),
        ("vis_words", _c_i64),
        ("scale", ctypes.c_float),
    ]


# name -> (restype, argtypes)
_SIGNATURES = {
    "ddt_last_error": (ctypes.c_char_p, []),
    "ddt_abi_version": (ctypes.c_int, []),
    "ddt_sm_count": (ctypes.c_int, [ctypes.c_int]),
    "ddt_launch_count": (ctypes.c_uint64, []),
    "ddt_tree_build_workspace_size": (ctypes.c_size_t, [_c_i64, _c_i64, _c_i64]),
    "ddt_tree_build": (ctypes.c_int, [_c_p, ctypes.c_int, _c_i64, _c_i64, _c_i64, _c_i64, _c_p, _c_i64,
                                      ctypes.POINTER(TreeOutputs), _c_p, ctypes.c_size_t, _c_p]),
    "ddt_tree_build_noalloc": (ctypes.c_int, [_c_p, ctypes.c_int, _c_i64, _c_i64, _c_i64, _c_i64, _c_p, _c_i64,
                                              ctypes.POINTER(TreeOutputs), _c_p]),
    "ddt_tree_from_log_probs": (ctypes.c_int, [_c_p, _c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_i64,
                                               ctypes.POINTER(TreeOutputs), _c_p]),
    "ddt_tree_mask_fill": (ctypes.c_int, [_c_p, ctypes.c_int, _c_i64, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_i64,
                                          _c_i64, ctypes.c_double, _c_p]),
    "ddt_mask_to_bits": (ctypes.c_int, [_c_p, ctypes.c_int, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_p]),
    "ddt_tree_attention_workspace_size": (ctypes.c_size_t, [_c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_int]),
    "ddt_tree_attention": (ctypes.c_int, [ctypes.POINTER(AttentionArgs), _c_p, ctypes.c_size_t, _c_p]),
    "ddt_sample_rows_workspace_size": (ctypes.c_size_t, [ctypes.c_int64, ctypes.c_int64]),
    "ddt_sample_rows": (ctypes.c_int, [_c_p, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                       ctypes.c_float, ctypes.c_uint64, ctypes.c_uint64, _c_p, _c_p, ctypes.c_size_t,
                                       _c_p]),
    "ddt_tree_attention_window": (ctypes.c_int, [ctypes.POINTER(AttentionArgs), _c_p, _c_p, ctypes.c_size_t, _c_p]),
    "ddt_tree_attention_f32": (ctypes.c_int, [ctypes.POINTER(AttentionArgs), _c_p, _c_p, _c_p]),
    "ddt_tree_attention_dev": (ctypes.c_int, [ctypes.POINTER(AttentionArgs), _c_p, _c_p, _c_p, _c_p,
                                              ctypes.c_size_t, _c_p]),
    "ddt_kv_append": (ctypes.c_int, [_c_p, _c_p, _c_i64, _c_i64, _c_p, _c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
                                     _c_i64, _c_p, _c_p, _c_p]),
    "ddt_rms_norm": (ctypes.c_int, [_c_p, ctypes.c_int, _c_i64, _c_p, _c_p, _c_i64, _c_i64, _c_i64, ctypes.c_float,
                                    _c_p]),
    "ddt_qk_norm_rope_append": (ctypes.c_int, [ctypes.c_int, _c_p, _c_i64, _c_p, _c_p, _c_i64, _c_i64, _c_p, _c_p,
                                               _c_i64, _c_i64, _c_p, _c_p, ctypes.c_float, ctypes.c_float, _c_p, _c_p,
                                               _c_i64, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_p, _c_p, _c_i64,
                                               _c_i64, _c_i64, _c_p, _c_p]),
    "ddt_silu_mul": (ctypes.c_int, [_c_p, _c_p, _c_p, ctypes.c_int, _c_i64, _c_p]),
    "ddt_silu_mul_rows": (ctypes.c_int, [_c_p, _c_p, _c_i64, _c_p, _c_i64, _c_i64, _c_i64, ctypes.c_int, _c_p]),
    "ddt_wgemm_workspace_size": (ctypes.c_size_t, [_c_i64, _c_i64, _c_i64]),
    "ddt_wgemm": (ctypes.c_int, [_c_p, _c_i64, _c_i64, _c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_p, _c_i64, _c_i64,
                                 _c_p, ctypes.c_size_t, _c_p]),
    "ddt_wgemm_gate_up": (ctypes.c_int, [_c_p, _c_i64, _c_i64, _c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_i64, _c_p,
                                         ctypes.c_size_t, _c_p]),
    "ddt_wgemm_head_stats_size": (ctypes.c_size_t, [_c_i64, _c_i64]),
    "ddt_wgemm_head": (ctypes.c_int, [_c_p, _c_i64, _c_i64, _c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_p,
                                      ctypes.c_size_t, _c_p, ctypes.c_size_t, _c_p]),
    "ddt_tree_build_head": (ctypes.c_int, [_c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_p, _c_i64,
                                           ctypes.POINTER(TreeOutputs), _c_p, ctypes.c_size_t, _c_p]),
    "ddt_set_pdl": (ctypes.c_int, [ctypes.c_int]),
    "ddt_tree_accept_workspace_size": (ctypes.c_size_t, [_c_i64, _c_i64]),
    "ddt_tree_accept": (ctypes.c_int, [_c_p, ctypes.c_int, _c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_p, _c_p,
                                       _c_i64, _c_p, _c_p, ctypes.c_size_t, _c_p]),
    "ddt_tree_walk": (ctypes.c_int, [_c_p, _c_i64, _c_p, _c_p, _c_p, _c_p, _c_i64, _c_p, _c_p]),
    "ddt_argmax_rows": (ctypes.c_int, [_c_p, ctypes.c_int, _c_i64, _c_i64, _c_i64, _c_p, _c_p, ctypes.c_size_t,
                                       _c_p]),
    "ddt_tree_commit": (ctypes.c_int, [_c_p, _c_i64, _c_p, _c_i64, _c_p, _c_p, _c_i64, _c_i64, _c_p, _c_i64, _c_i64,
                                       _c_p, _c_i64, _c_p]),
    "ddt_kv_compact": (ctypes.c_int, [_c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_p, _c_p,
                                      _c_i64, _c_p]),
    "ddt_eagle3_accept": (ctypes.c_int, [_c_p, ctypes.c_int, _c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_i64, _c_i64,
                                         _c_p, _c_p, _c_p, _c_p, ctypes.c_size_t, _c_p]),
}

_lib = None
_lock = threading.Lock()


class DDTreeError(RuntimeError):
    """A C-ABI entry point returned an error status."""


def load():
    """Load (and bind) the native library; raises if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise ImportError(
                    f"{LIB_PATH.name} is not built; run `python -m ddtree_eagle3_patch_b200.build` "
                    "(the B200 path has no CPU fallback)")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def exported_symbols():
    return list(_SIGNATURES)


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = load().ddt_last_error().decode(errors="replace")
        raise DDTreeError(f"{what} failed (status {rc}): {msg}")


def ptr(t) -> int:
    return 0 if t is None else t.data_ptr()


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return DDT_F32
    if dt == torch.bfloat16:
        return DDT_BF16
    if dt == torch.float16:
        return DDT_F16
    if dt == torch.bool:
        return DDT_BOOL
    raise TypeError(f"unsupported dtype {dt}")


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def raw_stream(index: int) -> int:
    """Current CUDA stream handle of device `index` (the cheap form of
    stream_of, used on per-layer paths where the wrapper's host time counts)."""
    if _raw_stream is not None:
        return _raw_stream(index)
    return torch.cuda.current_stream(index).cuda_stream


def require_cuda(t: torch.Tensor, name: str) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor on the B200 path (got {getattr(t, 'device', type(t))})")


class Workspaces:
    """Zero-initialised, grow-only device scratch buffers per (kind, device).

    The tree-build and accept kernels keep self-resetting counters in their
    workspace, so a buffer is zero-filled once when allocated and reused."""

    def __init__(self):
        self._bufs: dict = {}

    def get(self, kind: str, device: torch.device, nbytes: int) -> torch.Tensor:
        key = (kind, device.index if device.index is not None else torch.cuda.current_device())
        buf = self._bufs.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.zeros(max(int(nbytes), 256), dtype=torch.uint8, device=device)
            self._bufs[key] = buf
        return buf

    def current(self, kind: str, index: int):
        """The buffer of (kind, device index) as it stands, or None."""
        return self._bufs.get((kind, index))


WORKSPACES = Workspaces()
