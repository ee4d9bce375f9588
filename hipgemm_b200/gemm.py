"""Torch-facing wrappers of the C ABI (device memory and streams come from torch;
the arithmetic runs in the sm_100a kernels of libhipgemm_b200.so).

    C = fp8_gemm_tn(A, B, scale_a, scale_b)    # C[M,N] bf16 = sa*sb * A[M,K] . B[N,K]^T

mirrors the reference operator fp8_gemm_4wave_256x256x128<M,N,K>(A, B_T, C)
(nirw4nna/hipgemm fp8_4wave.hpp:334-338): same operand order and layouts, with the
per-tensor scales of the benchmark configs added and any M, N % 8, K % 16 accepted.
"""
from __future__ import annotations

import ctypes

import torch

from ._lib import HgemmError, check, lib

_FP8_DTYPES = (torch.uint8, torch.float8_e4m3fn)


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream_handle(stream: torch.cuda.Stream | None, device_index: int | None = None) -> int | None:
    if stream is not None:
        return stream.cuda_stream or None
    if device_index is not None and _raw_stream is not None:
        return _raw_stream(device_index) or None  # no Python Stream object on the hot path
    return torch.cuda.current_stream().cuda_stream or None


# torch's raw current-stream and current-device queries (plain ints); absent in some builds,
# then the public API.
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)
_get_device = getattr(torch._C, "_cuda_getDevice", None)
_fns: dict[str, object] = {}


def _fn(name: str):
    """The C function `name`, looked up once."""
    f = _fns.get(name)
    if f is None:
        f = _fns[name] = getattr(lib(), name)
    return f


class _on_device:
    """Makes `index` the current CUDA device for the call, entering torch's device context
    only when it is not already current (the common case costs one query)."""

    def __init__(self, index: int):
        self.ctx = None if torch.cuda.current_device() == index else torch.cuda.device(index)

    def __enter__(self):
        if self.ctx is not None:
            self.ctx.__enter__()

    def __exit__(self, *exc):
        if self.ctx is not None:
            self.ctx.__exit__(*exc)
        return False


def _check_operand(name: str, t: torch.Tensor) -> None:
    if t.dtype not in _FP8_DTYPES:
        raise TypeError(f"{name} must be float8_e4m3fn or uint8 (e4m3 bits), got {t.dtype}")
    if t.dim() != 2 or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous 2-D tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be on a CUDA device (there is no CPU path)")


def _check_scale(name: str, s: torch.Tensor | None, device: torch.device) -> None:
    if s is None:
        return
    if s.dtype != torch.float32 or s.numel() != 1 or s.device != device:
        raise ValueError(f"{name} must be a 1-element float32 tensor on {device}")


def _scale_ptr(name: str, s: torch.Tensor | None, dev: int) -> int | None:
    """The device pointer of a per-tensor scale on CUDA device `dev` (None = 1.0)."""
    if s is None:
        return None
    if s.dtype != torch.float32 or s.numel() != 1 or s.get_device() != dev:
        raise ValueError(f"{name} must be a 1-element float32 tensor on cuda:{dev}")
    return s.data_ptr()


def fp8_gemm_tn(a: torch.Tensor, b: torch.Tensor, scale_a: torch.Tensor | None = None,
                scale_b: torch.Tensor | None = None, out: torch.Tensor | None = None, *, config: int = 0,
                schedule: int = 0, workspace: torch.Tensor | None = None,
                stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """C[M,N] (bf16) = scale_a * scale_b * a[M,K] @ b[N,K]^T, fp32 accumulation.

    config: tile configuration (0 = automatic, see config_names()); schedule: 0 automatic
    (may pick split-K over CTA clusters for skinny problems with long K: reproducible bits, but
    not those of the whole-K kernels), 1 data-parallel only (whole-K tiles: the same bits for
    any tiling), 2 stream-K; workspace: optional caller-owned device buffer for a stream-K
    schedule (else the library's stream-ordered pool is used)."""
    # The common case is checked with a few cheap integer and dtype tests (this wrapper's host
    # time adds to every launch of a small GEMM); anything unusual takes the detailed checks,
    # which raise the specific error.
    dev = a.get_device()
    if (dev < 0 or b.get_device() != dev or a.dtype not in _FP8_DTYPES or b.dtype not in _FP8_DTYPES
            or a.dim() != 2 or b.dim() != 2 or not a.is_contiguous() or not b.is_contiguous()):
        _check_operand("a", a)
        _check_operand("b", b)
        raise ValueError("a and b must be on the same device")
    M, K = a.shape
    N, Kb = b.shape
    if Kb != K:
        raise ValueError(f"K mismatch: a is {tuple(a.shape)}, b is {tuple(b.shape)}")
    sa = _scale_ptr("scale_a", scale_a, dev)
    sb = _scale_ptr("scale_b", scale_b, dev)
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    elif (out.dtype != torch.bfloat16 or out.dim() != 2 or out.shape[0] != M or out.shape[1] != N
          or not out.is_contiguous()):
        raise ValueError("out must be a contiguous (M, N) bfloat16 tensor")
    ws_ptr, ws_bytes = None, 0
    if workspace is not None:
        if workspace.get_device() != dev or not workspace.is_contiguous():
            raise ValueError("workspace must be a contiguous tensor on the operands' device")
        ws_ptr, ws_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
    f = _fns.get("hgemm_fp8_tn_ex") or _fn("hgemm_fp8_tn_ex")
    if _get_device is not None and stream is None and _raw_stream is not None and _get_device() == dev:
        rc = f(a.data_ptr(), b.data_ptr(), out.data_ptr(), M, N, K, sa, sb, _raw_stream(dev) or None,
               int(config), int(schedule), ws_ptr, ws_bytes)
    else:
        with _on_device(dev):
            rc = f(a.data_ptr(), b.data_ptr(), out.data_ptr(), M, N, K, sa, sb, _stream_handle(stream, dev),
                   int(config), int(schedule), ws_ptr, ws_bytes)
    if rc:
        check(rc, "hgemm_fp8_tn")
    return out


def plan(M: int, N: int, K: int, config: int = 0, schedule: int = 0, device=None) -> dict:
    """The launch plan the library would use on `device` (default: current)."""
    out = (ctypes.c_int * 6)()
    with torch.cuda.device(device if device is not None else torch.cuda.current_device()):
        check(lib().hgemm_plan(M, N, K, config, schedule, out), "hgemm_plan")
        nbytes = ctypes.c_size_t(0)
        check(lib().hgemm_workspace_bytes(M, N, K, config, schedule, ctypes.byref(nbytes)), "hgemm_workspace_bytes")
    from ._lib import config_names
    return {"config": config_names()[out[0]], "grid": out[1], "tiles": out[2], "dp_tiles": out[3],
            "sk_tiles": out[4], "sk_slots": out[5], "workspace_bytes": int(nbytes.value)}


def fp8_gemm_tn_rows(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor, row_begin: int, row_end: int,
                     scale_a: torch.Tensor | None = None, scale_b: torch.Tensor | None = None,
                     stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """Rows [row_begin, row_end) of fp8_gemm_tn(a, b) written into the same rows of `out`."""
    _check_operand("a", a)
    _check_operand("b", b)
    M, K = a.shape
    N = b.shape[0]
    if out.dtype != torch.bfloat16 or tuple(out.shape) != (M, N) or not out.is_contiguous():
        raise ValueError("out must be a contiguous (M, N) bfloat16 tensor")
    with _on_device(a.device.index):
        rc = _fn("hgemm_fp8_tn_rows")(_ptr(a), _ptr(b), _ptr(out), M, N, K, int(row_begin), int(row_end),
                                     _ptr(scale_a), _ptr(scale_b), _stream_handle(stream, a.device.index))
    check(rc, "hgemm_fp8_tn_rows")
    return out


def device_status() -> int:
    """Reads and clears the current device's kernel status word (0 = healthy)."""
    v = ctypes.c_uint32(0)
    rc = lib().hgemm_device_status(ctypes.byref(v))
    if rc not in (0, -6):
        raise HgemmError(rc, "hgemm_device_status")
    return int(v.value)


# ---- host utilities (utils.hpp mirror) -------------------------------------------------

def host_init_random(n: int, seed: int = 0, mean: float = -1.0, stddev: float = 1.0) -> torch.Tensor:
    """utils.hpp:27-33: mt19937(seed) -> normal_distribution<float>(mean, stddev) -> e4m3.
    Returns n e4m3 bytes in a CPU uint8 tensor (defaults are the reference's)."""
    out = torch.empty(n, dtype=torch.uint8)
    lib().hgemm_host_init_random(out.data_ptr(), n, seed, mean, stddev)
    return out


def host_make_quantized(n: int, seed: int, mean: float = 0.0, stddev: float = 1.0,
                        out: torch.Tensor | None = None) -> tuple[torch.Tensor, float]:
    """Per-tensor amax/448 quantisation of n seeded N(mean, stddev) draws (CPU)."""
    if out is None:
        out = torch.empty(n, dtype=torch.uint8)
    scale = lib().hgemm_host_make_quantized(out.data_ptr(), n, seed, mean, stddev)
    return out, float(scale)


def quantize_e4m3(x: torch.Tensor, out: torch.Tensor | None = None, scale: torch.Tensor | None = None,
                  stream: torch.cuda.Stream | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-tensor e4m3 quantisation on the GPU (hgemm_quantize_e4m3): returns (q, scale)
    with scale = amax(|x|)/448 as a 1-element float32 tensor and q = e4m3(x / scale) as
    uint8 bits of x's shape, ready for fp8_gemm_tn."""
    if not x.is_cuda or not x.is_contiguous():
        raise ValueError("x must be a contiguous CUDA tensor (there is no CPU path)")
    if x.dtype == torch.float32:
        dt = 0
    elif x.dtype == torch.bfloat16:
        dt = 1
    else:
        raise TypeError(f"x must be float32 or bfloat16, got {x.dtype}")
    if out is None:
        out = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    if scale is None:
        scale = torch.empty(1, dtype=torch.float32, device=x.device)
    if out.numel() != x.numel() or out.dtype != torch.uint8 or not out.is_contiguous():
        raise ValueError("out must be a contiguous uint8 tensor with x's size")
    with _on_device(x.device.index):
        rc = _fn("hgemm_quantize_e4m3")(x.data_ptr(), dt, x.numel(), out.data_ptr(), scale.data_ptr(),
                                       _stream_handle(stream, x.device.index))
    check(rc, "hgemm_quantize_e4m3")
    return out, scale


def quantize_e4m3_delayed(x: torch.Tensor, scale_in: torch.Tensor, out: torch.Tensor | None = None,
                          amax_out: torch.Tensor | None = None,
                          stream: torch.cuda.Stream | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Delayed-scaling e4m3 quantisation in one pass (hgemm_quantize_e4m3_delayed): returns
    (q, amax) with q = e4m3(x / scale_in) and amax = max|x| of this x (1-element float32), from
    which the caller forms the next scale (e.g. amax / 448)."""
    if not x.is_cuda or not x.is_contiguous():
        raise ValueError("x must be a contiguous CUDA tensor (there is no CPU path)")
    if x.dtype == torch.float32:
        dt = 0
    elif x.dtype == torch.bfloat16:
        dt = 1
    else:
        raise TypeError(f"x must be float32 or bfloat16, got {x.dtype}")
    _check_scale("scale_in", scale_in, x.device)
    if scale_in is None:
        raise ValueError("scale_in is required")
    if out is None:
        out = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    if amax_out is None:
        amax_out = torch.empty(1, dtype=torch.float32, device=x.device)
    if out.numel() != x.numel() or out.dtype != torch.uint8 or not out.is_contiguous():
        raise ValueError("out must be a contiguous uint8 tensor with x's size")
    with _on_device(x.device.index):
        rc = _fn("hgemm_quantize_e4m3_delayed")(x.data_ptr(), dt, x.numel(), out.data_ptr(), scale_in.data_ptr(),
                                               amax_out.data_ptr(), _stream_handle(stream, x.device.index))
    check(rc, "hgemm_quantize_e4m3_delayed")
    return out, amax_out


def fp8_gemm_tn_from_host(a_host: torch.Tensor, b_host: torch.Tensor, c_host: torch.Tensor,
                          scales_host: torch.Tensor | None, d_a: torch.Tensor, d_b: torch.Tensor, d_c: torch.Tensor,
                          d_scales: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """C = sa*sb * A . B^T from host tensors into a host tensor, with the copies in and out
    overlapped with the GEMMs (hgemm_fp8_tn_from_host).  a_host (M, K) and b_host (N, K)
    uint8 e4m3 bits, c_host (M, N) bfloat16, scales_host 2 float32 (or None) -- all on
    the CPU, ideally pinned; d_a, d_b, d_c, d_scales: device buffers of the same shapes."""
    M, K = a_host.shape
    N = b_host.shape[0]
    for name, t in (("a_host", a_host), ("b_host", b_host), ("c_host", c_host)):
        if t.is_cuda or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous CPU tensor")
    if c_host.dtype != torch.bfloat16 or tuple(c_host.shape) != (M, N):
        raise ValueError("c_host must be an (M, N) bfloat16 tensor")
    if tuple(d_c.shape) != (M, N) or d_c.dtype != torch.bfloat16:
        raise ValueError("d_c must be an (M, N) bfloat16 CUDA tensor")
    if scales_host is not None and (scales_host.numel() != 2 or scales_host.dtype != torch.float32 or d_scales is None):
        raise ValueError("scales_host must hold 2 float32 values, with a 2-float d_scales")
    with torch.cuda.device(d_c.device):
        rc = lib().hgemm_fp8_tn_from_host(a_host.data_ptr(), b_host.data_ptr(), c_host.data_ptr(), M, N, K,
                                          _ptr(scales_host), d_a.data_ptr(), d_b.data_ptr(), d_c.data_ptr(),
                                          _ptr(d_scales), _stream_handle(stream))
    check(rc, "hgemm_fp8_tn_from_host")
    return c_host


def mx_sf_to_blocked(sf: torch.Tensor, K: int) -> torch.Tensor:
    """Row-major e8m0 scale factors (rows x K/32, uint8, CPU) -> the blocked layout the MX
    kernel reads (hgemm_host_mx_sf_to_blocked); returns a CPU uint8 tensor."""
    if sf.is_cuda or sf.dtype != torch.uint8 or sf.dim() != 2 or sf.shape[1] * 32 != K:
        raise ValueError("sf must be a CPU uint8 (rows, K/32) tensor")
    sf = sf.contiguous()
    rows = sf.shape[0]
    out = torch.empty(int(lib().hgemm_mx_sf_bytes(rows, K)), dtype=torch.uint8)
    check(lib().hgemm_host_mx_sf_to_blocked(sf.data_ptr(), rows, K, out.data_ptr()), "hgemm_host_mx_sf_to_blocked")
    return out


def fp8_gemm_tn_mx(a: torch.Tensor, b: torch.Tensor, sfa_blocked: torch.Tensor, sfb_blocked: torch.Tensor,
                   scale_a: torch.Tensor | None = None, scale_b: torch.Tensor | None = None,
                   out: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None,
                   config: int = 0) -> torch.Tensor:
    """OCP MX e4m3 GEMM (one e8m0 scale per 32 K elements of each row of a and b, blocked
    layout from mx_sf_to_blocked, on the device): C = sa*sb * sum_k (a 2^sfa)(b 2^sfb).
    config: 0 chooses by wave count, 1 = 128 x 256 tiles, 2 = 128 x 128 tiles, 3 = 256 x 256
    tiles on CTA pairs; 4 and 5 = configs 3 and 2 with two K blocks per TMA load (K % 128 == 0,
    else HgemmError)."""
    _check_operand("a", a)
    _check_operand("b", b)
    M, K = a.shape
    N = b.shape[0]
    for name, t, rows in (("sfa_blocked", sfa_blocked, M), ("sfb_blocked", sfb_blocked, N)):
        if not t.is_cuda or t.dtype != torch.uint8 or t.numel() < int(lib().hgemm_mx_sf_bytes(rows, K)):
            raise ValueError(f"{name} must be a CUDA uint8 tensor of hgemm_mx_sf_bytes({rows}, {K}) bytes")
    _check_scale("scale_a", scale_a, a.device)
    _check_scale("scale_b", scale_b, a.device)
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    dev = a.device.index
    with _on_device(dev):
        rc = _fn("hgemm_fp8_tn_mx_config")(a.data_ptr(), b.data_ptr(), out.data_ptr(), M, N, K,
                                           sfa_blocked.data_ptr(), sfb_blocked.data_ptr(), _ptr(scale_a),
                                           _ptr(scale_b), config, _stream_handle(stream, dev))
    if rc:
        check(rc, "hgemm_fp8_tn_mx_config")
    return out


def quantize_mx_e4m3(x: torch.Tensor, out: torch.Tensor | None = None, sf_out: torch.Tensor | None = None,
                     stream: torch.cuda.Stream | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """OCP MX e4m3 quantisation on the GPU (hgemm_quantize_mx_e4m3) of a rows x K fp32 or bf16
    tensor: returns (q, sf_blocked), q the e4m3 bits (uint8, x's shape) and sf_blocked the
    e8m0 scales in the layout fp8_gemm_tn_mx takes (also torch._scaled_mm's blocked e8m0
    layout)."""
    if not x.is_cuda or not x.is_contiguous() or x.dim() != 2:
        raise ValueError("x must be a contiguous 2-D CUDA tensor (there is no CPU path)")
    if x.dtype == torch.float32:
        dt = 0
    elif x.dtype == torch.bfloat16:
        dt = 1
    else:
        raise TypeError(f"x must be float32 or bfloat16, got {x.dtype}")
    rows, K = x.shape
    sf_bytes = int(lib().hgemm_mx_sf_bytes(rows, K))
    q = torch.empty((rows, K), dtype=torch.uint8, device=x.device) if out is None else out
    sf = torch.empty(sf_bytes, dtype=torch.uint8, device=x.device) if sf_out is None else sf_out
    if q.numel() != x.numel() or q.dtype != torch.uint8 or not q.is_contiguous() or q.device != x.device:
        raise ValueError("out must be a contiguous uint8 tensor with x's size on x's device")
    if sf.numel() < sf_bytes or sf.dtype != torch.uint8 or not sf.is_contiguous() or sf.device != x.device:
        raise ValueError(f"sf_out must be a contiguous uint8 tensor of {sf_bytes} bytes on x's device")
    with _on_device(x.device.index):
        rc = _fn("hgemm_quantize_mx_e4m3")(x.data_ptr(), dt, rows, K, q.data_ptr(), sf.data_ptr(),
                                          _stream_handle(stream, x.device.index))
    check(rc, "hgemm_quantize_mx_e4m3")
    return q, sf
