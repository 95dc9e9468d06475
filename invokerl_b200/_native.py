"""ctypes binding of ``libinvokerl_b200.so``, the C ABI declared in ``include/invokerl_b200.h``.

The library is built in-tree by ``python -m invokerl_b200.csrc.build`` (nvcc, sm_100a).  There
is no CPU or PyTorch fallback: if the library is missing, or a tensor is not on a CUDA device,
every op raises.
"""

from __future__ import annotations

import ctypes
import os
import threading
from ctypes import POINTER, c_double, c_float, c_int32, c_int64, c_size_t, c_uint8, c_void_p
from pathlib import Path

import torch

# The in-tree build; INVOKERL_B200_LIBRARY may point at another build of the same ABI.
LIB_PATH = Path(os.environ.get("INVOKERL_B200_LIBRARY") or Path(__file__).resolve().with_name("libinvokerl_b200.so"))

IKRL_DTYPE_F32 = 0
IKRL_DTYPE_BF16 = 1
IKRL_KL_SCHULMAN = 0
IKRL_KL_SIMPLE = 1
IKRL_KL_NONE = 2
IKRL_LOSS_GRPO = 0
IKRL_LOSS_PPO = 1
# Launch knobs of ikrl_set_tuning (include/invokerl_b200.h, IKRL_TUNE_*).
TUNE = {
    "cta_pairs": 0,
    "skip_zero_rows": 1,
    "wide": 2,
    "persistent": 3,
    "pace": 4,
    "pace_kb": 5,
    "pace_lag": 6,
    "balance_splits": 7,
    "l2_policy": 8,
    "l2_budget_mb": 9,
    "loss_kernel": 10,
    "pace_kb_long": 11,
    "split_tail": 12,
    "dh_split_k": 13,
}
TUNE_DEFAULT = -(1 << 63)
LOSS_NSUMS = 16
LOSS_NMETRICS = 12
SIMPO_NMETRICS = 8

_ERR_NAMES = {
    1: "invalid argument",
    2: "alignment",
    3: "unsupported",
    4: "workspace",
    5: "CUDA error",
    6: "device error",
}


class IkrlError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, name: str, code: int, msg: str):
        super().__init__(f"{name} failed ({_ERR_NAMES.get(code, code)}): {msg}")
        self.code = code


class LossParams(ctypes.Structure):
    _fields_ = [
        ("family", c_int32),
        ("ratio_lo", c_float),
        ("ratio_hi", c_float),
        ("clip_metric_eps", c_float),
        ("beta", c_float),
        ("kl_type", c_int32),
        ("entropy_coef", c_float),
        ("vf_coef", c_float),
        ("vf_clip_eps", c_float),
    ]


# name -> (restype, argtypes).  Pointers are passed as c_void_p (device addresses).
_P = c_void_p
_SIGNATURES: dict[str, tuple] = {
    "ikrl_last_error": (ctypes.c_char_p, []),
    "ikrl_abi_version": (ctypes.c_int, []),
    "ikrl_launch_count": (ctypes.c_ulonglong, []),
    "ikrl_mask_count": (ctypes.c_int, [_P, c_int64, _P, _P]),
    "ikrl_broadcast_advantages": (ctypes.c_int, [_P, _P, c_int32, c_int32, _P, _P]),
    "ikrl_group_advantages": (
        ctypes.c_int,
        [_P, _P, _P, c_int32, c_int32, c_int32, c_int32, c_float, _P, _P, _P],
    ),
    "ikrl_token_group_advantages": (ctypes.c_int, [_P, _P, c_int32, c_int32, c_int32, _P, _P]),
    "ikrl_masked_moments_workspace_bytes": (c_size_t, [c_int64]),
    "ikrl_masked_moments": (ctypes.c_int, [_P, _P, c_int64, _P, _P, c_size_t, _P]),
    "ikrl_gae_advantages": (
        ctypes.c_int,
        [_P, _P, _P, _P, c_int32, c_int32, c_float, c_float, _P, _P],
    ),
    "ikrl_clip_loss_workspace_bytes": (c_size_t, [c_int64]),
    "ikrl_clip_loss_fwd": (
        ctypes.c_int,
        [_P, c_int32, _P, _P, _P, _P, _P, c_int32, c_int32, c_int32, _P, _P, _P, _P,
         POINTER(LossParams), _P, _P, _P, _P, c_size_t, _P],
    ),
    "ikrl_clip_loss_finalize": (ctypes.c_int, [_P, _P, POINTER(LossParams), _P, _P, _P]),
    "ikrl_scale_grad": (ctypes.c_int, [_P, c_int32, c_int64, _P, _P]),
    "ikrl_simpo_workspace_bytes": (c_size_t, [c_int32]),
    "ikrl_simpo_fwd": (
        ctypes.c_int,
        [_P, c_int32, _P, _P, c_int32, c_int32, c_float, c_float, c_int32, _P, _P, _P, _P,
         c_size_t, _P],
    ),
    "ikrl_simpo_bwd": (ctypes.c_int, [_P, _P, c_int32, c_int32, _P, _P, c_int32, _P]),
    "ikrl_dpo_workspace_bytes": (c_size_t, [c_int32]),
    "ikrl_dpo_fwd": (
        ctypes.c_int,
        [_P, c_int32, _P, _P, _P, c_int32, c_int32, c_float, c_float, c_int32, _P, _P, _P, _P, c_size_t, _P],
    ),
    "ikrl_logits_logprob_fwd": (
        ctypes.c_int,
        [_P, c_int64, _P, c_int64, c_int32, _P, _P, _P, _P],
    ),
    "ikrl_logits_logprob_bwd": (
        ctypes.c_int,
        [_P, c_int64, _P, _P, _P, c_int64, c_int32, _P, c_int64, _P],
    ),
    "ikrl_lmhead_fwd_workspace_bytes": (c_size_t, [c_int64, c_int32, c_int32]),
    "ikrl_lmhead_logprob_fwd": (
        ctypes.c_int,
        [_P, _P, _P, c_int64, c_int32, c_int32, _P, _P, _P, c_size_t, _P],
    ),
    "ikrl_lmhead_bwd_workspace_bytes": (c_size_t, [c_int64, c_int32, c_int32, c_int64, c_int32, c_int32]),
    "ikrl_lmhead_logprob_bwd": (
        ctypes.c_int,
        [_P, _P, _P, _P, _P, c_int64, c_int32, c_int32, c_int64, _P, _P, c_int32, c_int32, _P, c_size_t, _P],
    ),
    "ikrl_lmhead_status": (ctypes.c_int, [_P, POINTER(c_int32), _P]),
    "ikrl_lmhead_cache_row_elems": (ctypes.c_int, [c_int32, POINTER(c_int64), POINTER(c_int64)]),
    "ikrl_lmhead_cache_fwd_workspace_bytes": (c_size_t, [c_int64, c_int32, c_int32]),
    "ikrl_lmhead_logprob_fwd_cached": (
        ctypes.c_int,
        [_P, _P, _P, c_int64, c_int32, c_int32, _P, _P, _P, c_int64, _P, _P, _P, _P, c_size_t, _P],
    ),
    "ikrl_lmhead_logprob_bwd_cached": (
        ctypes.c_int,
        [_P, _P, _P, _P, _P, c_int64, c_int32, c_int32, c_int64, _P, _P, c_int32, c_int32, _P, _P, _P, _P,
         c_size_t, _P],
    ),
    "ikrl_lmhead_set_cta_pairs": (ctypes.c_int, [c_int32]),
    "ikrl_lmhead_plan": (ctypes.c_int, [c_int32, c_int64, c_int32, c_int32, c_int32, POINTER(c_int32)]),
    "ikrl_lmhead_logprob_fwd_noalloc": (
        ctypes.c_int,
        [_P, _P, _P, c_int64, c_int32, c_int32, _P, _P, _P],
    ),
    "ikrl_lmhead_noalloc_status": (ctypes.c_int, [POINTER(c_int32), _P]),
    "ikrl_set_tuning": (ctypes.c_int, [c_int32, c_int64, POINTER(c_int64)]),
    "ikrl_get_tuning": (ctypes.c_int, [c_int32, POINTER(c_int64)]),
    "ikrl_lmhead_shard_fwd": (
        ctypes.c_int,
        [_P, _P, _P, c_int64, c_int32, c_int32, c_int64, _P, _P, _P, c_size_t, _P],
    ),
    "ikrl_vocab_parallel_combine": (ctypes.c_int, [_P, _P, c_int64, c_int32, c_int64, _P, _P, _P]),
    "ikrl_lmhead_shard_bwd": (
        ctypes.c_int,
        [_P, _P, _P, _P, _P, c_int64, c_int32, c_int32, c_int64, c_int64, _P, _P, c_int32, c_int32, _P, c_size_t,
         _P],
    ),
    "ikrl_pack_rollouts": (
        ctypes.c_int,
        [_P, _P, _P, _P, _P, _P, c_int32, c_int32, c_int64, _P, _P, _P, _P, _P, _P],
    ),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """Load the native library once; raise if it was not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"invokerl_b200 native library not found at {LIB_PATH}; build it with "
                "`python -m invokerl_b200.csrc.build` (nvcc, sm_100a). There is no CPU fallback."
            )
        handle = ctypes.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | os.RTLD_LOCAL)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(handle, name, None)
            if fn is None:  # symbols added by later sources are bound lazily in bind()
                continue
            fn.restype = res
            fn.argtypes = args
        _lib = handle
        return handle


def bind(name: str, restype, argtypes) -> None:
    """Register the signature of an extra exported function."""
    _SIGNATURES[name] = (restype, argtypes)
    if _lib is not None:
        fn = getattr(_lib, name)
        fn.restype = restype
        fn.argtypes = argtypes


def exported_names() -> list[str]:
    return list(_SIGNATURES)


def call(name: str, *args) -> None:
    """Call a status-returning entry point; raise IkrlError on a non-zero status."""
    fn = getattr(lib(), name)
    rc = fn(*args)
    if rc != 0:
        msg = lib().ikrl_last_error()
        raise IkrlError(name, rc, msg.decode() if msg else "")


def set_tuning(knob: str, value: int | None) -> int:
    """Set a launch knob (None restores its default); returns the previous value."""
    prev = c_int64(0)
    call("ikrl_set_tuning", c_int32(TUNE[knob]), c_int64(TUNE_DEFAULT if value is None else int(value)),
         ctypes.byref(prev))
    return int(prev.value)


def get_tuning(knob: str) -> int:
    v = c_int64(0)
    call("ikrl_get_tuning", c_int32(TUNE[knob]), ctypes.byref(v))
    return int(v.value)


class tuning:
    """Context manager that sets launch knobs and restores their previous values on exit:
    ``with tuning(pace=0, wide=1): ...``."""

    def __init__(self, **knobs: int | None):
        self.knobs = knobs
        self.prev: dict[str, int] = {}

    def __enter__(self):
        for k, v in self.knobs.items():
            self.prev[k] = set_tuning(k, v)
        return self

    def __exit__(self, *exc):
        for k, v in self.prev.items():
            set_tuning(k, v)
        return False


# ---- tensor helpers -------------------------------------------------------------------------


def ptr(t: torch.Tensor | None) -> c_void_p | None:
    return None if t is None else c_void_p(t.data_ptr())


def require_cuda(*tensors: torch.Tensor | None, names: str = "") -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(
                f"invokerl_b200 runs on CUDA tensors only (got a {t.device} tensor{' ' + names if names else ''}); "
                "there is no CPU path"
            )
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} and {t.device}")
    if dev is None:
        raise RuntimeError("no CUDA tensor given")
    return dev


def stream_of(device: torch.device) -> c_void_p:
    return c_void_p(torch.cuda.current_stream(device).cuda_stream)


def dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return IKRL_DTYPE_F32
    if t.dtype == torch.bfloat16:
        return IKRL_DTYPE_BF16
    raise TypeError(f"unsupported dtype {t.dtype}; expected float32 or bfloat16")


def as_mask(m: torch.Tensor) -> torch.Tensor:
    """Bool/uint8 mask as a contiguous byte tensor (a view for bool, no copy)."""
    m = m.contiguous()
    if m.dtype == torch.bool:
        return m.view(torch.uint8)
    if m.dtype == torch.uint8:
        return m
    return (m != 0).view(torch.uint8)


_ws_cache: dict[tuple[int, int], torch.Tensor] = {}


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """A per-(device, stream) byte workspace grown on demand.  Calls on one stream are ordered,
    so reusing the buffer across calls of that stream is safe."""
    key = (device.index if device.index is not None else torch.cuda.current_device(),
           torch.cuda.current_stream(device).cuda_stream)
    buf = _ws_cache.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
        _ws_cache[key] = buf
    return buf


def f32(x: float) -> c_float:
    return c_float(float(x))


def i32(x: int) -> c_int32:
    return c_int32(int(x))


def i64(x: int) -> c_int64:
    return c_int64(int(x))


def sz(x: int) -> c_size_t:
    return c_size_t(int(x))


__all__ = [
    "IkrlError",
    "LossParams",
    "lib",
    "call",
    "bind",
    "ptr",
    "require_cuda",
    "stream_of",
    "dtype_code",
    "as_mask",
    "workspace",
    "set_tuning",
    "get_tuning",
    "tuning",
    "c_double",
    "c_uint8",
    "c_int32",
    "byref",
]

byref = ctypes.byref
