"""W8A8 GS128 GEMM on B200 tensor cores (drop-in for ksdraft/kernels/gemm.py:53).

`w8a8_gemm(a_codes, a_scales, w_codes, w_scales, group)` keeps the reference
signature, checks and padding (gemm.py:60-74) and returns fp32 (M, N).  The
work runs in `ksd8_w8a8_gemm`: tcgen05 kind::i8 MMAs fed by TMA, an int32
accumulator per 128-wide K group in TMEM, and the fp32 group sum
acc = fmaf(RN(float(dot_g) * sa), sw, acc) in the epilogue.

`gemm_out` is the internal form used by the fused cells: output dtype
(fp32/bf16/fp16), a row-stride, an optional fp32 bias, fp16 saturation and a
non-finite flag (the FP16 gradient handoff of ks3_int8.py:75-84).
"""

from __future__ import annotations

import torch

from .. import _lib
from .quant import GROUP_SIZE, SCALE_DTYPE, _check_group  # noqa: F401 (reference names)


class GemmTimer:
    """Records a CUDA event pair around every GEMM launch while active
    (on the launching stream); used by bench.py for the roofline figures.
    With external=True the events may be recorded during CUDA-graph capture:
    each replay of the graph then re-records them, and durations_ms() after a
    replay gives that replay's GEMM times."""

    active: "GemmTimer | None" = None

    def __init__(self, external: bool = False):
        self.external = external
        self.pairs: list[tuple[torch.cuda.Event, torch.cuda.Event, int]] = []

    def __enter__(self):
        GemmTimer.active = self
        return self

    def __exit__(self, *exc):
        GemmTimer.active = None

    def durations_ms(self) -> list[tuple[float, int]]:
        torch.cuda.synchronize()
        return [(s.elapsed_time(e), ops) for s, e, ops in self.pairs]


def _aligned(t: torch.Tensor) -> torch.Tensor:
    """Contiguous and 16-byte aligned (TMA base-address rule)."""
    if not t.is_contiguous() or t.data_ptr() % 16:
        t = t.contiguous() if not t.is_contiguous() else t.clone()
    return t


def gemm_out(a_codes: torch.Tensor, a_scales: torch.Tensor, w_codes: torch.Tensor,
             w_scales: torch.Tensor, *, out: torch.Tensor | None = None,
             out_dtype: torch.dtype = torch.float32, bias: torch.Tensor | None = None,
             clamp_f16: bool = False, status: torch.Tensor | None = None,
             round_f16: bool = False, if_status: bool = False) -> torch.Tensor:
    """Y = A W^T with GS128 scales; K must already be a multiple of 128.

    round_f16 (fp32 `out`): store float(fp16(Y)) and flag overflow in `status`
    (the FP16 gradient handoff written into an fp32 buffer).  if_status: the
    launch does nothing unless `status` is already non-zero on the device."""
    _lib.require_cuda(a_codes, a_scales, w_codes, w_scales)
    M, K = a_codes.shape
    N = w_codes.shape[0]
    a_codes, w_codes = _aligned(a_codes), _aligned(w_codes)
    a_scales, w_scales = a_scales.contiguous(), w_scales.contiguous()
    if out is None:
        out = torch.empty(M, N, dtype=out_dtype, device=a_codes.device)
    flags = 0
    if bias is not None:
        bias = bias.float().contiguous()
        flags |= _lib.EPI_BIAS
    if clamp_f16:
        flags |= _lib.EPI_CLAMP_F16
    if status is not None and not if_status:
        flags |= _lib.EPI_FLAG_NONFINITE
    if round_f16:
        flags |= _lib.EPI_ROUND_F16
    if if_status:
        if status is None:
            raise ValueError("if_status needs a status tensor")
        flags |= _lib.EPI_IF_STATUS
    timer = GemmTimer.active if not if_status else None  # predicated launches are not timed
    if timer is not None:
        ev0 = torch.cuda.Event(enable_timing=True, external=timer.external)
        ev1 = torch.cuda.Event(enable_timing=True, external=timer.external)
        ev0.record()
    rc = _lib.lib().ksd8_w8a8_gemm(
        a_codes.data_ptr(), a_scales.data_ptr(), w_codes.data_ptr(), w_scales.data_ptr(), M, N, K,
        GROUP_SIZE, out.data_ptr(), _lib.dtype_code(out), out.stride(0) if M > 1 else N,
        _lib.ptr(bias), flags, _lib.ptr(status), _lib.stream_ptr(a_codes.device))
    if timer is not None:
        ev1.record()
        timer.pairs.append((ev0, ev1, 2 * M * N * K))
    _lib.check(rc, "w8a8_gemm")
    return out


def _validate_and_pad(a_codes, a_scales, w_codes, w_scales, group):
    """Reference checks and partial-group padding (ksdraft/kernels/gemm.py:60-74)."""
    M, K = a_codes.shape
    if w_codes.shape[1] != K:
        raise ValueError(f"K mismatch: A {K} vs W {w_codes.shape[1]}")
    n_groups = a_scales.shape[-1]
    if w_scales.shape[-1] != n_groups:
        raise ValueError(f"scale group mismatch: A {n_groups} vs W {w_scales.shape[-1]}")
    Kp = n_groups * group
    if Kp < K:
        raise ValueError(f"K {K} exceeds the scales' padded length {Kp}")
    if K < Kp:
        a_codes = torch.nn.functional.pad(a_codes, (0, Kp - K))
        w_codes = torch.nn.functional.pad(w_codes, (0, Kp - K))
    return a_codes, w_codes


def w8a8_gemm(a_codes: torch.Tensor, a_scales: torch.Tensor,
              w_codes: torch.Tensor, w_scales: torch.Tensor,
              group: int = GROUP_SIZE) -> torch.Tensor:
    """(M,K)x(N,K)^T -> (M,N) fp32, inputs as produced by quantize_last_dim."""
    _check_group(group)
    a_codes, w_codes = _validate_and_pad(a_codes, a_scales, w_codes, w_scales, group)
    return gemm_out(a_codes, a_scales, w_codes, w_scales)


def w8a8_group_partials(a_codes: torch.Tensor, w_codes: torch.Tensor) -> torch.Tensor:
    """Per-group int32 dot products (G, M, N) of the same tensor-core main loop."""
    _lib.require_cuda(a_codes, w_codes)
    M, K = a_codes.shape
    N = w_codes.shape[0]
    if K % GROUP_SIZE:
        raise ValueError("K must be a multiple of 128")
    a_codes, w_codes = _aligned(a_codes), _aligned(w_codes)
    out = torch.empty(K // GROUP_SIZE, M, N, dtype=torch.int32, device=a_codes.device)
    rc = _lib.lib().ksd8_w8a8_group_partials(
        a_codes.data_ptr(), w_codes.data_ptr(), M, N, K, out.data_ptr(), None,
        _lib.stream_ptr(a_codes.device))
    _lib.check(rc, "w8a8_group_partials")
    return out
