"""ctypes binding of libokc_b200.so (the C ABI declared in include/okc_b200.h).

There is no fallback: if the library is missing or was built without sm_100a code the
import of okc_b200.ops fails with an error that says so.  Build it with
``python -m okc_b200.build``.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("OKC_B200_LIB", _PKG / "_lib" / "libokc_b200.so"))

OKC_OK = 0
OKC_ERR_INVALID = -1
OKC_ERR_ALIGNMENT = -2
OKC_ERR_WORKSPACE = -3
OKC_ERR_LAUNCH = -4
OKC_ERR_DEVICE = -5
OKC_ERR_TOO_LARGE = -6
ERR_NAMES = {
    OKC_ERR_INVALID: "invalid argument or unsupported shape",
    OKC_ERR_ALIGNMENT: "pointer or leading dimension not 16-byte aligned",
    OKC_ERR_WORKSPACE: "workspace too small",
    OKC_ERR_LAUNCH: "CUDA launch failed",
    OKC_ERR_DEVICE: "no sm_100a device or kernel image",
    OKC_ERR_TOO_LARGE: "request exceeds the fixed scratch of the no-alloc entry point",
}
DEVERR_TIMEOUT, DEVERR_PAGE, DEVERR_INDEX = 1, 2, 4

_p, _i, _f, _sz, _i64 = C.c_void_p, C.c_int, C.c_float, C.c_size_t, C.c_int64

# name -> (restype, argtypes); must match include/okc_b200.h
SIGNATURES: dict[str, tuple] = {
    "okc_version": (C.c_char_p, []),
    "okc_read_device_error": (_i, [_p, _p]),
    "okc_gemm_bf16_workspace_bytes": (_sz, [_i, _i, _i]),
    "okc_gemm_bf16": (_i, [_p, _i, _p, _i, _p, _i, _p, _i, _i, _i, _i, _p, _sz, _p]),
    "okc_gemm_bf16_ex": (_i, [_p, _i, _p, _i, _p, _i, _p, _i, _i, _i, _i, _i, _i, _p, _sz, _p]),
    "okc_rmsnorm_bf16": (_i, [_p, _i, _p, _p, _i, _i, _i, _f, _i, _p]),
    "okc_rope_kv_append": (_i, [_p, _i, _p, _p, _i, _i, _p, _p, _p, _p, _p, _p, _p,
                                _i, _i, _i, _i, _i, _i64, _p, _sz, _p]),
    "okc_gemm_bf16_rope_kv_append": (_i, [_p, _i, _p, _i, _i, _i, _i, _p, _p, _i, _i, _p, _p, _p, _p, _p, _p, _p,
                                          _i, _i, _i, _i, _i64, _f, _p, _sz, _p]),
    "okc_rope_kv_append_ex": (_i, [_p, _i, _p, _p, _i, _i, _p, _p, _p, _p, _p, _p, _p,
                                   _i, _i, _i, _i, _i, _i64, _f, _i, _f, _p, _sz, _p]),
    "okc_attn_decode_workspace_bytes": (_sz, [_i, _i, _i, _i, _i]),
    "okc_attn_decode_fp8_gated": (_i, [_p, _i, _p, _p, _p, _i, _p, _p, _p, _p, _i,
                                       _i, _i, _i, _i, _i, _i64, _f, _i, _p, _i, _f, _p, _sz, _p]),
    "okc_attn_decode_fp8_ex": (_i, [_p, _i, _p, _p, _p, _i, _p, _p, _p, _p, _i,
                                    _i, _i, _i, _i, _i, _i64, _f, _i, _i, _i, _p, _i, _f, _p, _sz, _p]),
    "okc_attn_prefill_fp8": (_i, [_p, _i, _p, _p, _p, _i, _i, _p, _p, _p, _p, _i, _f, _p, _i, _i, _i, _i, _i, _i,
                                  _i, _i64, _f, _i, _p, _sz, _p]),
    "okc_attn_decode_fp8": (_i, [_p, _i, _p, _p, _p, _i, _p, _p, _p, _p, _i,
                                 _i, _i, _i, _i, _i, _i64, _f, _i, _p, _sz, _p]),
    "okc_gemv_bf16": (_i, [_p, _p, _p, _i, _i, _i, _i, _p, _p]),
    "okc_kv_append_rope": (_i, [_p, _i, _p, _p, _i, _i, _p, _p, _p, _p, _p, _p, _p,
                                _i, _i, _i, _i, _i, _i64, _p, _sz, _p]),
    "okc_moe_w4a16": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _i,
                           _p, _sz, _p]),
    "okc_rmsnorm": (_i, [_p, _p, _p, _i, _i, _f, _p]),
    "okc_ipc_alloc": (_i, [_sz, C.POINTER(_p)]),
    "okc_ipc_free": (_i, [_p]),
    "okc_ipc_handle": (_i, [_p, _p]),
    "okc_ipc_open": (_i, [_p, C.POINTER(_p)]),
    "okc_ipc_close": (_i, [_p]),
    "okc_tp_allreduce_residual": (_i, [C.POINTER(_p), C.POINTER(_p), C.POINTER(_p), _p, _p, _i, _i, C.c_longlong,
                                       _p, _p]),
    "okc_tp_oproj_plan": (_i, [_i, _i, _i, _i, C.POINTER(_sz), C.POINTER(_i)]),
    "okc_tp_oproj_allreduce_residual": (_i, [_p, _i, _p, _i, _i, _i, _i, C.POINTER(_p), C.POINTER(_p),
                                             C.POINTER(_p), _p, _i, _p, _i, _i, _p, _p]),
    "okc_attn_decode_fp8_noalloc": (_i, [_p, _i, _p, _p, _p, _i, _p, _p, _p, _p, _i,
                                         _i, _i, _i, _i, _i, _i64, _f, _i, _p]),
    "okc_attn_decode_fp8_noalloc_error": (_i, [_p]),
    "okc_moe_route": (_i, [_p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _p]),
    "okc_moe_permute": (_i, [_p, _i, _i, _i, _i, _i, _p, _p, _p, _p, _i, _p]),
    "okc_moe_experts_workspace_bytes": (_sz, [_i, _i, _i, _i]),
    "okc_moe_experts_w4a16_ex": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _i,
                                      _i, _p, _sz, _p]),
    "okc_moe_experts_w4a16_post": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _i,
                                        _i, _p, _f, _p, _sz, _p]),
    "okc_residual_boundary": (_i, [_p, _p, _i, _p, _p, _p, _p, _p, _p, _p, _i, _i, _f, _f, _p]),
    "okc_moe_route_sigmoid": (_i, [_p, _i, _p, _p, _p, _p, _p, _i, _i, _i, _f, _f, _f, _p]),
    "okc_router_logits_workspace_bytes": (_sz, [_i, _i, _i]),
    "okc_router_logits": (_i, [_p, _i, _p, _p, _i, _i, _i, _i, _p, _sz, _p]),
    "okc_moe_experts_w4a16": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p,
                                   _i, _i, _i, _i, _i, _i, _p, _sz, _p]),
}

_lib = None


class OkcError(RuntimeError):
    pass


def load() -> C.CDLL:
    """Loads the library once; raises OkcError (never falls back) when it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise OkcError(f"{LIB_PATH} is missing: build it with `python -m okc_b200.build` "
                       "(the okc_b200 operators have no CPU fallback)")
    lib = C.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int, what: str) -> None:
    if status != OKC_OK:
        raise OkcError(f"{what}: {ERR_NAMES.get(status, 'error')} (status {status})")
