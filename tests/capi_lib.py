"""ctypes binding of libpersona_bgmv.so for the tests (the C ABI in
include/persona_bgmv.h).  Tensors are passed by data pointer; the stream is
torch's current CUDA stream."""

import ctypes
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
LIB_PATH = ROOT / "multi-lora-llm-kernel_b200" / "persona" / "libpersona_bgmv.so"
HEADERS = sorted((ROOT / "include").glob("*.h"))

F16, BF16 = 0, 1
REUSE_PLAN = 1

_p, _i64, _i32, _sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t

SIGNATURES = {
    "persona_status_string": (ctypes.c_char_p, [_i32]),
    "persona_abi_version": (_i32, []),
    "persona_bgmv_workspace_size": (_sz, [_i64]),
    "persona_bgmv_plan": (_i32, [_p, _i64, _i64, _p, _sz, _p, _p]),
    "persona_bgmv_shrink": (_i32, [_p, _i64, _p, _i64, _i64, _p, _p, _i64, _i64, _i64, _i64, _i32,
                                   _p, _sz, _i32, _p, _p]),
    "persona_bgmv_expand": (_i32, [_p, _p, _i64, _p, _p, _i64, _i64, _i64, _i64, _i64, _i32, _p, _sz,
                                   _i32, _p, _p]),
    "persona_bgmv_fused": (_i32, [_p, _i64, _p, _i64, _i64, _p, _i64, _p, _p, _i64, _i64, _i64, _i64,
                                  _i64, _i64, _i32, _p, _sz, _i32, _p, _p]),
    "persona_gemv_fp16": (_i32, [_p, _p, _p, _i64, _i64, _p]),
    "persona_bgmv_multi_workspace_size": (_sz, [_i64, _i32]),
    "persona_bgmv_fused_multi": (_i32, [_p, _i32, _p, _i64, _i64, _i64, _i32, _p, _sz, _i32, _p, _p]),
    "persona_bgmv_fused_noalloc": (_i32, [_p, _i64, _p, _i64, _i64, _p, _i64, _p, _p, _i64, _i64, _i64, _i64,
                                          _i64, _i64, _i32, _p, _p]),
    "persona_sgmv_workspace_size": (_sz, [_i64]),
    "persona_sgmv_shrink": (_i32, [_p, _i64, _p, _i64, _i64, _p, _p, _i64, _p, _i64, _i64, _i64, _i64, _i32,
                                   _p, _sz, _p, _p]),
    "persona_sgmv_expand": (_i32, [_p, _p, _i64, _p, _p, _i64, _p, _i64, _i64, _i64, _i64, _i64, _i32, _p, _sz,
                                   _p, _p]),
    "persona_sgmv_fused": (_i32, [_p, _i64, _p, _i64, _i64, _p, _i64, _p, _p, _i64, _p, _i64, _i64, _i64, _i64,
                                  _i64, _i64, _i32, _p, _sz, _p, _p]),
    "persona_nf4_packed_bytes": (_sz, [_i64, _i64]),
    "persona_nf4_quantize_workspace_size": (_sz, [_i64, _i64]),
    "persona_nf4_quantize": (_i32, [_p, _i64, _i64, _i64, _p, _p, _p, _sz, _p]),
    "persona_nf4_dequantize": (_i32, [_p, _p, _i64, _i64, _p, _i64, _p]),
    "persona_nf4_linear_workspace_size": (_sz, [_p, _i32]),
    "persona_nf4_linear": (_i32, [_p, _i32, _i64, _p, _sz, _p, _p]),
}


class Nf4Problem(ctypes.Structure):
    """persona_nf4_problem (include/persona_bgmv.h)."""
    _fields_ = [("packed", _p), ("offset", _p), ("x", _p), ("ldx", _i64), ("y", _p), ("ldy", _i64), ("N", _i64),
                ("K", _i64)]


class Problem(ctypes.Structure):
    """persona_bgmv_problem (include/persona_bgmv.h)."""
    _fields_ = [("x", _p), ("ldx", _i64), ("a_pool", _p), ("a_slot_stride", _i64), ("a_row_stride", _i64),
                ("b_pool", _p), ("b_slot_stride", _i64), ("y", _p), ("ldy", _i64), ("K", _i64), ("N", _i64)]


def declared_symbols():
    """Function names declared in include/*.h."""
    names = set()
    for h in HEADERS:
        text = h.read_text()
        names.update(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(persona_\w+)\s*\(", text, re.M))
    return names


_LIB = None


def load():
    global _LIB
    if _LIB is None:
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            f = getattr(lib, name)
            f.restype = res
            f.argtypes = args
        _LIB = lib
    return _LIB


def check(status):
    if status != 0:
        raise RuntimeError(f"persona C ABI status {status}: {load().persona_status_string(status).decode()}")
