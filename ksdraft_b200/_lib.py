"""ctypes binding of libksd8.so (the C ABI declared in include/ksd8.h).

The library is loaded lazily on first use.  There is no fallback: if the
shared object is missing, or a tensor handed to an op is not a CUDA tensor,
the op raises.  Status codes are mapped to the exceptions the reference
raises for the same conditions (ValueError for shapes, TypeError for dtypes).
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libksd8.so"

OK, ERR_SHAPE, ERR_ALIGN, ERR_DTYPE, ERR_LAUNCH, ERR_TIMEOUT, ERR_UNSUPPORTED, ERR_ARG, \
    ERR_NONFINITE = range(9)
ERR_SCRATCH_LIMIT = 9
VJP_STATIC_MAX_PARTIALS = 1 << 21

F32, F16, BF16, I8 = 0, 1, 2, 3
Q_ROUND_F16, Q_DITHER, Q_PLAIN_LOADS = 1, 2, 8
GRAD_CLIP_SCRATCH = 592  # KSD8_GRAD_CLIP_SCRATCH
EPI_CLAMP_F16, EPI_BIAS, EPI_FLAG_NONFINITE, EPI_ROUND_F16, EPI_IF_STATUS = 1, 2, 4, 8, 16
NL = {"fp32": 0, "fp16": 1, "int8": 2}

_DT = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16, torch.int8: I8}

i64, i32, u64, f32, vp = C.c_int64, C.c_int, C.c_uint64, C.c_float, C.c_void_p

# name -> argtypes (restype is always int)
SIGNATURES: dict[str, list] = {
    "ksd8_version": [],
    "ksd8_status_string": [i32],
    "ksd8_last_cuda_error": [],
    "ksd8_sm_count": [i32],
    "ksd8_quantize_rows": [vp, i32, i64, i64, i64, i32, i32, f32, u64, u64, vp, i64, vp, vp, vp],
    "ksd8_quantize_cols": [vp, i32, vp, i32, i64, i64, i64, i32, i32, vp, i64, vp, vp, vp],
    "ksd8_w8a8_gemm": [vp, vp, vp, vp, i64, i64, i64, i32, vp, i32, i64, vp, i32, vp, vp],
    "ksd8_w8a8_group_partials": [vp, vp, i64, i64, i64, vp, vp, vp],
    "ksd8_ks3_pack": [vp, vp, vp, i64, vp, vp, vp, vp, vp, vp, vp, vp],
    "ksd8_ks3_spine_quant": [vp, i64, i64, vp, vp, vp, vp, vp, vp, vp, i32, vp, vp, vp, vp,
                             vp],
    "ksd8_ks3_spine_table": [i64, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp],
    "ksd8_ks3_vjp": [vp, vp, i64, i64, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp],
    "ksd8_ks3_vjp_reduce": [vp, i64, i64, vp, vp, vp, vp, vp, vp, vp],
    "ksd8_ks3_vjp_reduce_f32": [vp, i64, i64, vp, vp, vp, vp, vp, vp, vp],
    "ksd8_rosa_pack_bits": [vp, i32, i64, i64, i64, i64, i64, i64, vp, vp, vp],
    "ksd8_rosa_credits": [vp, vp, vp, i64, i64, i32, vp, vp, vp, vp, vp, vp],
    "ksd8_rosa_match": [vp, vp, vp, i64, i64, i64, i32, vp, vp, i32, i64, i64, i64, vp, vp, vp,
                        vp],
    "ksd8_rosa_match_scratch": [vp, vp, vp, i64, i64, i64, i32, vp, vp, i32, i64, i64, i64, vp,
                                vp, vp, i64, vp, vp],
    "ksd8_rosa_timemix_quantize": [vp, i32, i64, i64, i64, vp, vp, vp, vp, vp, vp, vp, vp, vp,
                                   vp, vp],
    "ksd8_adamw_step": [vp, vp, i32, vp, vp, i64, f32, f32, f32, f32, f32, i32, vp, vp],
    "ksd8_adamw_step_scaled": [vp, vp, i32, vp, vp, i64, f32, f32, f32, f32, f32, i32, vp, vp, vp],
    "ksd8_grad_clip_coef": [vp, i64, f32, vp, vp, vp, vp],
    "ksd8_adamw_multi": [i32, vp, vp, i32, vp, vp, vp, f32, f32, f32, f32, f32, i32, vp, vp, vp],
    "ksd8_philox_uniform": [u64, u64, i64, vp, vp],
    "ksd8_fp16_tanh_table": [i64, vp, vp],
    "ksd8_dspine_ln_fwd": [vp, vp, vp, i32, i64, i64, vp, vp, vp, f32, vp, vp, vp, vp, vp, vp],
    "ksd8_dspine_ln_bwd": [vp, vp, vp, vp, vp, vp, vp, i32, i64, i64, vp, vp, vp, vp, vp, vp,
                           i64, vp, vp],
    "ksd8_transfer_rows": [vp, i32, vp, i64, i64, vp, vp, vp, vp, vp],
    "ksd8_transfer_bwd": [vp, i32, vp, vp, vp, i64, i64, f32, vp, vp, i64, vp, vp, vp, vp],
    "ksd8_rosa_payload_bwd": [vp, vp, vp, vp, i32, i64, i64, vp, i64, vp, vp],
    "ksd8_rosa_decode_build": [vp, i64, i64, i64, i32, vp, vp, vp, vp, i64, vp, vp],
    "ksd8_rosa_decode_merge": [vp, i64, i64, i64, i64, i32, vp, vp, vp, vp, vp, vp, i64, vp,
                               vp],
    "ksd8_rosa_decode_step": [vp, vp, vp, i32, i64, i64, i64, i64, i64, i32, vp, vp, vp, i64,
                              vp, vp, vp, vp, i64, vp, vp, i64, i32, vp, vp, i64, vp, vp, vp],
    "ksd8_rosa_set_algorithm": [i32],
    "ksd8_set_sm_reserve": [i32],
    "ksd8_get_sm_reserve": [],
    "ksd8_ce_partials": [vp, i32, i64, i64, i64, vp, i64, vp, vp, vp, vp, vp],
    "ksd8_ce_grad": [vp, i32, i64, i64, i64, vp, i64, vp, vp, f32, vp, i64, vp, vp],
    "ksd8_ce_grad_quant": [vp, i32, i64, i64, i64, vp, i64, vp, vp, f32, vp, i64, vp, vp, i64, vp,
                           vp, vp],
    "ksd8_topk_rows": [vp, i32, vp, i64, i64, i64, i32, i64, vp, vp, vp, vp],
    "ksd8_ks3_vjp_static": [vp, vp, i64, i64, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp,
                            vp, vp, vp, vp],
}

_lib: C.CDLL | None = None


def load() -> C.CDLL:
    """Load libksd8.so and declare every entry point's signature."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m ksdraft_b200.build` "
                "(ksdraft_b200 has no CPU fallback)")
        lib = C.CDLL(str(LIB_PATH))
        for name, argtypes in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = C.c_char_p if name == "ksd8_status_string" else C.c_int
        _lib = lib
    return _lib


def status_string(code: int) -> str:
    return load().ksd8_status_string(code).decode()


# Number of kernel-launching C-ABI calls made by this process (each compute
# entry point enqueues exactly one kernel); read by bench.py for gpu_launches.
LAUNCHES = 0


def check(rc: int, what: str) -> None:
    global LAUNCHES
    LAUNCHES += 1
    if rc == OK:
        return
    msg = f"{what}: {status_string(rc)}"
    if rc == ERR_SHAPE:
        raise ValueError(msg)
    if rc == ERR_DTYPE:
        raise TypeError(msg)
    if rc == ERR_LAUNCH:
        msg += f" (cudaError {load().ksd8_last_cuda_error()})"
    raise RuntimeError(msg)


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}") from None


def require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                "ksdraft_b200 ops run on CUDA tensors only (no CPU fallback); "
                f"got a tensor on {t.device}")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def lib() -> C.CDLL:
    return load()
