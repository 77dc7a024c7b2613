"""ctypes binding of libvitb200.so, the C ABI declared in include/vitb200.h.

The library is the product path: there is no fallback. Importing this module
raises ImportError when the library has not been built (run
``python vit-engine-cuda_b200/build.py`` or ``__graft_entry__.build()``).
The shared object itself is opened on the first call into it, so a process
that imports the package only for its host-side helpers (the seeded
synthetic weights of ``vit_cuda.weights``, say) never maps it.
"""
from __future__ import annotations

import ctypes
import os
import threading
from ctypes import POINTER, c_char_p, c_float, c_int, c_int64, c_size_t, c_void_p

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libvitb200.so")

# Status codes (include/vitb200.h).
OK = 0
E_INVALID_ARG = -1
E_UNSUPPORTED = -2
E_WORKSPACE = -3
E_DEVICE_TIMEOUT = -4
E_NO_TMA = -5
E_ALIGNMENT = -6

EPI_NONE = 0
EPI_BIAS = 1
EPI_BIAS_GELU = 2
EPI_BIAS_RESID = 3


class VitB200Error(RuntimeError):
    """A libvitb200 entry point returned a non-zero status."""

    def __init__(self, what: str, status: int):
        self.status = status
        super().__init__(f"{what}: {status_string(status)} (status {status})")


class BlockParams(ctypes.Structure):
    _fields_ = [(name, c_void_p) for name in (
        "norm1_w", "norm1_b", "qkv_w_pair", "qkv_b", "proj_w_pair", "proj_b",
        "norm2_w", "norm2_b", "fc1_w_pair", "fc1_b", "fc2_w_pair", "fc2_b")] + [
        ("qkv_w_f16", c_void_p), ("qkv_acc_scale", c_float),
        ("proj_w_f16", c_void_p), ("proj_acc_scale", c_float),
        ("fc1_w_f16", c_void_p), ("fc1_acc_scale", c_float),
        ("fc2_w_f16", c_void_p), ("fc2_acc_scale", c_float),
        ("attn_f16", c_int), ("q_scale", c_float), ("k_scale", c_float), ("v_scale", c_float),
        ("ln_qkv_w_f16", c_void_p), ("ln_qkv_acc_scale", c_float),
        ("ln_qkv_c", c_void_p), ("ln_qkv_d", c_void_p),
        ("ln_fc1_w_f16", c_void_p), ("ln_fc1_acc_scale", c_float),
        ("ln_fc1_c", c_void_p), ("ln_fc1_d", c_void_p)]


class VitParams(ctypes.Structure):
    _fields_ = [
        ("depth", c_int), ("embed_dim", c_int), ("num_heads", c_int), ("mlp_dim", c_int),
        ("patch", c_int), ("in_chans", c_int), ("img_h", c_int), ("img_w", c_int),
        ("num_classes", c_int), ("ln_eps", c_float), ("attn_scale", c_float),
        ("patch_w_pair", c_void_p), ("patch_b", c_void_p), ("cls_token", c_void_p),
        ("pos_embed", c_void_p), ("blocks", POINTER(BlockParams)),
        ("norm_w", c_void_p), ("norm_b", c_void_p),
        ("head_w_pair", c_void_p), ("head_b", c_void_p),
        ("patch_w_f16", c_void_p), ("patch_acc_scale", c_float),
        ("ln_fold", c_int),
    ]


_P = c_void_p
_SIGNATURES = {
    "vitb200_version": (c_int, []),
    "vitb200_status_string": (c_char_p, [c_int]),
    "vitb200_init": (c_int, []),
    "vitb200_device_error": (c_int, [POINTER(c_int), c_int]),
    "vitb200_num_sms": (c_int, []),
    "vitb200_launch_count": (ctypes.c_uint64, []),
    "vitb200_set_gemm_variant": (c_int, [c_int]),
    "vitb200_set_split_k": (c_int, [c_int]),
    "vitb200_set_gemm_split": (c_int, [c_int]),
    "vitb200_check_wait_timeout": (c_int, [c_int, _P]),
    "vitb200_gemm_plan": (c_int, [c_int64, c_int, c_int, c_int, POINTER(c_int), POINTER(c_int)]),
    "vitb200_split_tf32": (c_int, [_P, c_int64, c_int, c_int64, _P, c_int, _P]),
    "vitb200_split_f16": (c_int, [_P, c_int64, c_int, c_int64, c_float, _P, c_int64, c_int, _P]),
    "vitb200_gemm_f16": (c_int, [_P, _P, c_float, _P, _P, _P, c_int64, _P, c_int64, c_int, c_int,
                                 c_int, _P]),
    "vitb200_preprocess": (c_int, [_P, c_int, c_int, c_int, c_int64, c_int, c_int,
                                   POINTER(c_float), POINTER(c_float), _P, _P]),
    "vitb200_layernorm": (c_int, [_P, _P, _P, _P, c_int64, c_int, c_float, _P]),
    "vitb200_gemm_workspace_bytes": (c_size_t, [c_int64, c_int, c_int]),
    "vitb200_gemm": (c_int, [_P, _P, _P, _P, _P, c_int64, c_int, c_int, c_int, _P, c_size_t, _P]),
    "vitb200_gemm_noalloc": (c_int, [_P, _P, _P, _P, _P, c_int64, c_int, c_int, c_int, _P]),
    "vitb200_gemm_pairs": (c_int, [_P, _P, _P, _P, _P, c_int64, _P, c_int64, c_int, c_int, c_int,
                                   _P]),
    "vitb200_qkv_workspace_bytes": (c_size_t, [c_int64, c_int]),
    "vitb200_qkv": (c_int, [_P, _P, _P, _P, c_int64, c_int, _P, c_size_t, _P]),
    "vitb200_mlp_workspace_bytes": (c_size_t, [c_int64, c_int, c_int]),
    "vitb200_mlp": (c_int, [_P, _P, _P, _P, _P, _P, _P, c_int64, c_int, c_int, _P, c_size_t,
                            _P]),
    "vitb200_attention_workspace_bytes": (c_size_t, [c_int, c_int, c_int]),
    "vitb200_attention": (c_int, [_P, _P, _P, _P, c_int, c_int, c_int, c_int64, c_int64, c_int64,
                                  c_int64, c_float, _P, c_size_t, _P]),
    "vitb200_attention_f16_workspace_bytes": (c_size_t, [c_int, c_int, c_int]),
    "vitb200_attention_f16": (c_int, [_P, _P, _P, _P, c_int, c_int, c_int, c_int64, c_int64,
                                      c_int64, c_int64, c_float, c_float, c_float, _P, c_size_t,
                                      _P]),
    "vitb200_patch_embed_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int]),
    "vitb200_patch_embed": (c_int, [_P, _P, _P, _P, c_int, c_int, c_int, c_int, c_int, _P,
                                    c_size_t, _P]),
    "vitb200_pos_encoding": (c_int, [_P, _P, _P, _P, c_int, c_int, c_int, _P]),
    "vitb200_classifier_workspace_bytes": (c_size_t, [c_int, c_int, c_int]),
    "vitb200_classifier": (c_int, [_P, _P, _P, _P, c_int, c_int, c_int, c_int, _P, c_size_t,
                                   _P]),
    "vitb200_vit_workspace_bytes": (c_size_t, [POINTER(VitParams), c_int]),
    "vitb200_vit_forward": (c_int, [POINTER(VitParams), _P, _P, c_int, _P, c_size_t, _P]),
    "vitb200_vit_forward_features": (c_int, [POINTER(VitParams), _P, _P, c_int, _P, c_size_t,
                                             _P]),
    "vitb200_vit_embed": (c_int, [POINTER(VitParams), _P, _P, c_int, _P, c_size_t, _P]),
    "vitb200_vit_block": (c_int, [POINTER(VitParams), c_int, _P, c_int, _P, c_size_t, _P]),
    "vitb200_vit_head": (c_int, [POINTER(VitParams), _P, _P, _P, c_int, _P, c_size_t, _P]),
}


def _missing() -> ImportError:
    return ImportError(
        f"vit_cuda: {LIB_PATH} is missing; build it with "
        "`python vit-engine-cuda_b200/build.py` (there is no CPU fallback)")


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise _missing()
    cdll = ctypes.CDLL(LIB_PATH)
    for name, (restype, argtypes) in _SIGNATURES.items():
        fn = getattr(cdll, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return cdll


class _Library:
    """libvitb200.so, opened (and its signatures declared) on the first
    attribute access; each entry point is then cached on this object, so later
    calls cost a plain attribute lookup."""

    def __init__(self):
        self._cdll = None
        self._lock = threading.Lock()

    def _open(self) -> ctypes.CDLL:
        with self._lock:
            if self._cdll is None:
                self._cdll = _load()
            return self._cdll

    @property
    def loaded(self) -> bool:
        return self._cdll is not None

    def __getattr__(self, name: str):
        if name.startswith("__"):
            raise AttributeError(name)
        fn = getattr(self._open(), name)
        self.__dict__[name] = fn
        return fn


if not os.path.exists(LIB_PATH):
    raise _missing()
lib = _Library()


def status_string(status: int) -> str:
    return lib.vitb200_status_string(int(status)).decode()


def check(status: int, what: str) -> None:
    if status != 0:
        raise VitB200Error(what, status)


def exported_names() -> list[str]:
    return sorted(_SIGNATURES)


def device_error(clear: bool = True) -> int:
    """Synchronises the current device and returns (optionally clearing) its
    error word: 0, or the code of a kernel that gave up on a bounded wait."""
    code = c_int(0)
    check(lib.vitb200_device_error(ctypes.byref(code), 1 if clear else 0), "vitb200_device_error")
    return code.value


def set_split_k(enabled: bool) -> bool:
    """Switches split-K of the model's small block GEMMs (on by default; a
    batch-1 forward spreads each GEMM's K over more SMs). Off, an image's logits
    are bitwise the same in any batch of fewer than 1024 token rows; on, they
    agree to FP32 rounding. Affects later launches (not a captured graph).
    Returns the previous setting; process-wide."""
    return bool(lib.vitb200_set_split_k(1 if enabled else 0))


def set_gemm_split(ksplit: int) -> int:
    """Forces the K split of later small GEMM launches to `ksplit` wherever it
    fits (0: the automatic choice). For tuning and tests; returns the previous
    setting; process-wide."""
    return int(lib.vitb200_set_gemm_split(int(ksplit)))


def gemm_plan(M: int, K: int, N: int, f16: bool) -> tuple[int, int]:
    """(variant, ksplit) a GEMM of this shape launched now on the current
    device would use (vitb200_gemm_plan)."""
    v, d = c_int(0), c_int(0)
    check(lib.vitb200_gemm_plan(int(M), int(K), int(N), 1 if f16 else 0, ctypes.byref(v),
                                ctypes.byref(d)), "vitb200_gemm_plan")
    return v.value, d.value
