"""hipgemm_b200 — a B200-native (sm_100a) FP8 e4m3 TN GEMM with bf16 output.

C ABI: include/hipgemm_b200.h, implemented in csrc/ and built into
libhipgemm_b200.so (python -m hipgemm_b200.build).  This package binds it for
callers that hold their buffers in torch tensors, and adds the M-sharded
multi-GPU driver (shard.py).

GEMM:        fp8_gemm_tn (per-tensor scales), fp8_gemm_tn_rows (one rank's rows),
             fp8_gemm_tn_from_host (pinned host buffers, copies overlapped),
             fp8_gemm_tn_mx (OCP MX block scales), plan (the launch plan it would use).
Quantisers:  quantize_e4m3 (amax/448, two passes), quantize_e4m3_delayed (carried-over
             scale, one pass), quantize_mx_e4m3 (e8m0 per 32 elements, blocked scales),
             mx_sf_to_blocked (host conversion of row-major scales).
Host inputs: host_init_random, host_make_quantized (the reference harness's generator).
Status:      device_status (a kernel's bounded wait expired), HgemmError on negative codes.
"""
from ._lib import (HGEMM_ERR_ALIGNMENT, HGEMM_ERR_CUDA, HGEMM_ERR_DEVICE_TIMEOUT, HGEMM_ERR_INVALID_VALUE,
                   HGEMM_ERR_NO_DEVICE, HGEMM_ERR_UNSUPPORTED, HGEMM_OK, HGEMM_SCHEDULE_AUTO,
                   HGEMM_SCHEDULE_DATA_PARALLEL, HGEMM_SCHEDULE_STREAM_K, LIB_PATH, HgemmError, check, config_names,
                   lib)
from .gemm import (device_status, fp8_gemm_tn, fp8_gemm_tn_from_host, fp8_gemm_tn_mx, fp8_gemm_tn_rows,
                   host_init_random, host_make_quantized, mx_sf_to_blocked, plan, quantize_e4m3,
                   quantize_e4m3_delayed, quantize_mx_e4m3)

__all__ = [
    "HGEMM_OK", "HGEMM_ERR_INVALID_VALUE", "HGEMM_ERR_ALIGNMENT", "HGEMM_ERR_UNSUPPORTED", "HGEMM_ERR_CUDA",
    "HGEMM_ERR_NO_DEVICE", "HGEMM_ERR_DEVICE_TIMEOUT", "HGEMM_SCHEDULE_AUTO", "HGEMM_SCHEDULE_DATA_PARALLEL",
    "HGEMM_SCHEDULE_STREAM_K", "LIB_PATH", "HgemmError", "check", "config_names", "lib",
    "device_status", "fp8_gemm_tn", "fp8_gemm_tn_from_host", "fp8_gemm_tn_mx", "fp8_gemm_tn_rows",
    "host_init_random", "host_make_quantized", "mx_sf_to_blocked", "plan", "quantize_e4m3", "quantize_e4m3_delayed",
    "quantize_mx_e4m3",
]
