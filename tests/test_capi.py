"""CPU checks of the C ABI (no GPU needed): the library loads, exports every function
include/hipgemm_b200.h declares, rejects bad arguments before touching a device, and the
header-only drop-in for fp8_gemm_4wave_256x256x128<M,N,K> (fp8_4wave.hpp:334-338)
compiles as C++ and as plain C (the extern "C" part)."""
import ctypes
import os
import re
import subprocess

import pytest

import hipgemm_b200 as hg

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "hipgemm_b200.h")


def declared_functions() -> list[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(hgemm_\w+)\s*\(", text)) - {"hgemm_stream_t"})


def test_every_declared_symbol_is_exported():
    names = declared_functions()
    assert "hgemm_fp8_tn" in names and "hgemm_fp8_tn_rows" in names
    lib = ctypes.CDLL(hg.LIB_PATH)
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_library_metadata():
    L = hg.lib()
    assert L.hgemm_version().decode().startswith("hipgemm_b200")
    names = hg.config_names()
    assert names[0] == "auto" and {"bn256_s4", "pair256_s6", "bn128_s5_k2", "bn128_s5_k4"} <= set(names)
    assert L.hgemm_config_name(len(names)) is None
    for code in range(0, -7, -1):
        assert L.hgemm_error_string(code)


FAKE = 0x10000  # 16-byte aligned, never dereferenced: the checks fail before any CUDA call


@pytest.mark.parametrize("args,code", [
    ((FAKE, FAKE, FAKE, -1, 8, 16), hg.HGEMM_ERR_INVALID_VALUE),
    ((FAKE, FAKE, FAKE, 8, -8, 16), hg.HGEMM_ERR_INVALID_VALUE),
    ((FAKE, FAKE, FAKE, 8, 8, -16), hg.HGEMM_ERR_INVALID_VALUE),
    ((FAKE, FAKE, None, 8, 8, 16), hg.HGEMM_ERR_INVALID_VALUE),
    ((None, FAKE, FAKE, 8, 8, 16), hg.HGEMM_ERR_INVALID_VALUE),
    ((FAKE, None, FAKE, 8, 8, 16), hg.HGEMM_ERR_INVALID_VALUE),
    ((FAKE, FAKE, FAKE, 8, 8, 24), hg.HGEMM_ERR_ALIGNMENT),      # K % 16
    ((FAKE, FAKE, FAKE, 8, 12, 16), hg.HGEMM_ERR_ALIGNMENT),     # N % 8
    ((FAKE + 1, FAKE, FAKE, 8, 8, 16), hg.HGEMM_ERR_ALIGNMENT),  # misaligned A
    ((FAKE, FAKE + 8, FAKE, 8, 8, 16), hg.HGEMM_ERR_ALIGNMENT),  # misaligned B
    ((FAKE, FAKE, FAKE + 2, 8, 8, 16), hg.HGEMM_ERR_ALIGNMENT),  # misaligned C
    ((None, None, None, 0, 8, 16), hg.HGEMM_OK),                 # M == 0: nothing to do
    ((None, None, None, 8, 0, 16), hg.HGEMM_OK),                 # N == 0
])
def test_argument_checks_without_device(args, code):
    A, B, C, M, N, K = args
    assert hg.lib().hgemm_fp8_tn(A, B, C, M, N, K, None, None, None) == code


def test_config_and_row_range_checks():
    L = hg.lib()
    assert L.hgemm_fp8_tn_config(FAKE, FAKE, FAKE, 8, 8, 16, None, None, None, 99) == hg.HGEMM_ERR_INVALID_VALUE
    assert L.hgemm_fp8_tn_config(FAKE, FAKE, FAKE, 8, 8, 16, None, None, None, -1) == hg.HGEMM_ERR_INVALID_VALUE
    assert L.hgemm_fp8_tn_rows(FAKE, FAKE, FAKE, 8, 8, 16, 5, 3, None, None, None) == hg.HGEMM_ERR_INVALID_VALUE
    assert L.hgemm_fp8_tn_rows(FAKE, FAKE, FAKE, 8, 8, 16, 0, 9, None, None, None) == hg.HGEMM_ERR_INVALID_VALUE
    assert L.hgemm_fp8_tn_rows(FAKE, FAKE, FAKE, 8, 8, 16, -1, 3, None, None, None) == hg.HGEMM_ERR_INVALID_VALUE
    assert L.hgemm_fp8_tn_rows(FAKE, FAKE, FAKE, 8, 8, 16, 4, 4, None, None, None) == hg.HGEMM_OK


def test_python_wrapper_refuses_cpu_tensors():
    import torch
    a = torch.zeros((8, 16), dtype=torch.uint8)
    with pytest.raises(ValueError, match="CUDA"):
        hg.fp8_gemm_tn(a, a)
    with pytest.raises(TypeError):
        hg.fp8_gemm_tn(torch.zeros((8, 16), dtype=torch.float32), a)


def test_every_device_entry_point_refuses_cpu_tensors():
    """There is no CPU path: each torch-facing entry point raises before any CUDA call when
    handed host tensors (or host tensors where device buffers belong)."""
    import torch
    a = torch.zeros((8, 64), dtype=torch.uint8)
    x = torch.zeros((8, 64), dtype=torch.float32)
    sf = torch.zeros(hg.lib().hgemm_mx_sf_bytes(8, 64), dtype=torch.uint8)
    out = torch.empty((8, 8), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        hg.fp8_gemm_tn_rows(a, a, out, 0, 8)
    with pytest.raises(ValueError, match="CUDA"):
        hg.fp8_gemm_tn_mx(a, a, sf, sf)
    with pytest.raises(ValueError, match="CUDA"):
        hg.quantize_e4m3(x)
    with pytest.raises(ValueError, match="CUDA"):
        hg.quantize_e4m3_delayed(x, torch.ones(1))
    with pytest.raises(ValueError, match="CUDA"):
        hg.quantize_mx_e4m3(x)
    with pytest.raises(TypeError):
        hg.fp8_gemm_tn_mx(x, a, sf, sf)  # fp32 is not an e4m3 operand


def test_host_helpers_check_their_arguments():
    import torch
    a = torch.zeros((8, 64), dtype=torch.uint8)
    c = torch.empty((8, 8), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="c_host"):
        hg.fp8_gemm_tn_from_host(a, a, torch.empty((8, 9), dtype=torch.bfloat16), None, a, a, c)
    with pytest.raises(ValueError, match="d_c"):
        hg.fp8_gemm_tn_from_host(a, a, c, None, a, a, torch.empty((8, 9), dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="scales_host"):
        hg.fp8_gemm_tn_from_host(a, a, c, torch.ones(3), a, a, c)
    with pytest.raises(ValueError, match="sf"):
        hg.mx_sf_to_blocked(torch.zeros((8, 2), dtype=torch.float32), 64)
    with pytest.raises(ValueError, match="sf"):
        hg.mx_sf_to_blocked(torch.zeros((8, 3), dtype=torch.uint8), 64)  # K/32 columns expected


def test_header_compiles_as_cpp_and_c(tmp_path):
    cpp = tmp_path / "use.cpp"
    cpp.write_text(
        '#include "hipgemm_b200.h"\n'
        "int launch(const void* a, const void* b, void* c) {\n"
        "  return fp8_gemm_4wave_256x256x128<4096, 4096, 4096>(a, b, c);\n"
        "}\n")
    c = tmp_path / "use.c"
    c.write_text('#include "hipgemm_b200.h"\nint f(void) { return hgemm_fp8_tn(0, 0, 0, 0, 0, 0, 0, 0, 0); }\n')
    for cmd in (["g++", "-std=c++17", "-Wall", "-Werror", "-fsyntax-only", "-I", os.path.dirname(HEADER), str(cpp)],
                ["gcc", "-std=c99", "-Wall", "-Werror", "-fsyntax-only", "-I", os.path.dirname(HEADER), str(c)]):
        r = subprocess.run(cmd, capture_output=True, text=True)
        assert r.returncode == 0, r.stderr


def test_header_template_rejects_bad_shapes(tmp_path):
    cpp = tmp_path / "bad.cpp"
    cpp.write_text('#include "hipgemm_b200.h"\n'
                   "int f(const void* a, const void* b, void* c) {\n"
                   "  return fp8_gemm_4wave_256x256x128<256, 256, 200>(a, b, c);\n}\n")
    r = subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-I", os.path.dirname(HEADER), str(cpp)],
                       capture_output=True, text=True)
    assert r.returncode != 0 and "multiple of 16" in r.stderr


def test_fused_allgather_and_ipc_argument_checks():
    L = hg.lib()
    ptrs = (ctypes.c_void_p * 2)(FAKE, FAKE)
    bad = (ctypes.c_void_p * 2)(FAKE, None)
    mis = (ctypes.c_void_p * 2)(FAKE, FAKE + 2)
    args = (FAKE, FAKE)
    assert L.hgemm_fp8_tn_rows_allgather(*args, ptrs, 0, 0, 8, 8, 16, 0, 8, None, None, None) == hg.HGEMM_ERR_INVALID_VALUE
    assert L.hgemm_fp8_tn_rows_allgather(*args, ptrs, 9, 0, 8, 8, 16, 0, 8, None, None, None) == hg.HGEMM_ERR_INVALID_VALUE
    assert L.hgemm_fp8_tn_rows_allgather(*args, ptrs, 2, 2, 8, 8, 16, 0, 8, None, None, None) == hg.HGEMM_ERR_INVALID_VALUE
    assert L.hgemm_fp8_tn_rows_allgather(*args, None, 2, 0, 8, 8, 16, 0, 8, None, None, None) == hg.HGEMM_ERR_INVALID_VALUE
    assert L.hgemm_fp8_tn_rows_allgather(*args, bad, 2, 0, 8, 8, 16, 0, 8, None, None, None) == hg.HGEMM_ERR_INVALID_VALUE
    assert L.hgemm_fp8_tn_rows_allgather(*args, mis, 2, 0, 8, 8, 16, 0, 8, None, None, None) == hg.HGEMM_ERR_ALIGNMENT
    assert L.hgemm_fp8_tn_rows_allgather(*args, ptrs, 2, 0, 8, 8, 16, 5, 9, None, None, None) == hg.HGEMM_ERR_INVALID_VALUE
    assert L.hgemm_fp8_tn_rows_allgather(*args, ptrs, 2, 1, 8, 8, 16, 4, 4, None, None, None) == hg.HGEMM_OK
    assert L.hgemm_ipc_export(None, None, None) == hg.HGEMM_ERR_INVALID_VALUE
    assert L.hgemm_ipc_import(None, None) == hg.HGEMM_ERR_INVALID_VALUE
    assert L.hgemm_ipc_close(None) == hg.HGEMM_ERR_INVALID_VALUE


def test_quantiser_argument_checks():
    L = hg.lib()
    assert L.hgemm_quantize_e4m3(FAKE, 0, 16, FAKE, None, None) == hg.HGEMM_ERR_INVALID_VALUE
    assert L.hgemm_quantize_e4m3(None, 0, 16, FAKE, FAKE, None) == hg.HGEMM_ERR_INVALID_VALUE
    assert L.hgemm_quantize_e4m3(FAKE, 2, 16, FAKE, FAKE, None) == hg.HGEMM_ERR_INVALID_VALUE
    assert L.hgemm_quantize_e4m3(FAKE + 4, 0, 16, FAKE, FAKE, None) == hg.HGEMM_ERR_ALIGNMENT
    assert L.hgemm_quantize_e4m3(FAKE, 1, 16, FAKE + 8, FAKE, None) == hg.HGEMM_ERR_ALIGNMENT
    assert L.hgemm_quantize_e4m3(FAKE, 0, 16, FAKE, FAKE + 2, None) == hg.HGEMM_ERR_ALIGNMENT


def test_from_host_argument_checks():
    L = hg.lib()
    args = (FAKE, FAKE, FAKE)
    assert L.hgemm_fp8_tn_from_host(*args, -1, 8, 16, None, FAKE, FAKE, FAKE, None, None) == hg.HGEMM_ERR_INVALID_VALUE
    assert L.hgemm_fp8_tn_from_host(FAKE, FAKE, None, 8, 8, 16, None, FAKE, FAKE, FAKE, None, None) == \
        hg.HGEMM_ERR_INVALID_VALUE
    assert L.hgemm_fp8_tn_from_host(*args, 8, 8, 24, None, FAKE, FAKE, FAKE, None, None) == hg.HGEMM_ERR_ALIGNMENT
    assert L.hgemm_fp8_tn_from_host(*args, 8, 8, 16, FAKE, FAKE, FAKE, FAKE, None, None) == hg.HGEMM_ERR_INVALID_VALUE
    assert L.hgemm_fp8_tn_from_host(*args, 0, 8, 16, None, None, None, None, None, None) == hg.HGEMM_OK


def test_mx_argument_checks():
    L = hg.lib()
    sf = FAKE
    assert L.hgemm_mx_num_configs() == 6
    assert [L.hgemm_mx_config_name(c).decode() for c in range(6)] == ["auto", "mx_bn256_s4", "mx_bn128_s5",
                                                                       "mx_pair256_s6", "mx_pair256_s3x2",
                                                                       "mx_bn128_s3x2"]
    assert L.hgemm_mx_config_name(6) is None and L.hgemm_mx_config_name(-1) is None
    run = L.hgemm_fp8_tn_mx_config
    assert run(FAKE, FAKE, FAKE, 8, 8, 64, sf, sf, None, None, 6, None) == hg.HGEMM_ERR_INVALID_VALUE
    # Two K blocks per load: 128-byte K chunks only.
    assert run(FAKE, FAKE, FAKE, 8, 8, 160, sf, sf, None, None, 4, None) == hg.HGEMM_ERR_UNSUPPORTED
    assert run(FAKE, FAKE, FAKE, 8, 8, 96, sf, sf, None, None, 5, None) == hg.HGEMM_ERR_UNSUPPORTED
    assert run(FAKE, FAKE, FAKE, 8, 8, 64, sf, sf, None, None, -1, None) == hg.HGEMM_ERR_INVALID_VALUE
    assert run(FAKE, FAKE, FAKE, 8, 8, 48, sf, sf, None, None, 0, None) == hg.HGEMM_ERR_ALIGNMENT   # K % 32
    assert run(FAKE, FAKE, FAKE, 8, 8, 64, None, sf, None, None, 0, None) == hg.HGEMM_ERR_INVALID_VALUE
    assert run(FAKE, FAKE, FAKE, 8, 8, 64, sf + 4, sf, None, None, 0, None) == hg.HGEMM_ERR_ALIGNMENT
    assert run(FAKE, FAKE, FAKE, 8, 12, 64, sf, sf, None, None, 0, None) == hg.HGEMM_ERR_ALIGNMENT  # N % 8
    assert L.hgemm_fp8_tn_mx(FAKE, FAKE, FAKE, 0, 8, 64, None, None, None, None, None) == hg.HGEMM_OK
    assert L.hgemm_mx_sf_bytes(300, 1056) == 3 * 9 * 512 and L.hgemm_mx_sf_bytes(0, 64) == 0
    assert L.hgemm_host_mx_sf_to_blocked(FAKE, 4, 48, FAKE) == hg.HGEMM_ERR_INVALID_VALUE
    assert L.hgemm_host_mx_sf_to_blocked(None, 0, 64, None) == hg.HGEMM_OK  # empty: nothing touched


def test_mx_quantiser_argument_checks():
    L = hg.lib()
    q = L.hgemm_quantize_mx_e4m3
    assert q(FAKE, 2, 4, 64, FAKE, FAKE, None) == hg.HGEMM_ERR_INVALID_VALUE     # dtype
    assert q(FAKE, 0, -1, 64, FAKE, FAKE, None) == hg.HGEMM_ERR_INVALID_VALUE    # rows
    assert q(FAKE, 0, 4, 48, FAKE, FAKE, None) == hg.HGEMM_ERR_ALIGNMENT         # K % 32
    assert q(None, 0, 4, 64, FAKE, FAKE, None) == hg.HGEMM_ERR_INVALID_VALUE
    assert q(FAKE, 0, 4, 64, FAKE, None, None) == hg.HGEMM_ERR_INVALID_VALUE
    assert q(FAKE + 8, 1, 4, 64, FAKE, FAKE, None) == hg.HGEMM_ERR_ALIGNMENT
    assert q(FAKE, 0, 4, 64, FAKE + 4, FAKE, None) == hg.HGEMM_ERR_ALIGNMENT
    assert q(None, 0, 0, 64, None, None, None) == hg.HGEMM_OK                    # nothing to do


def test_delayed_quantiser_argument_checks():
    L = hg.lib()
    f = L.hgemm_quantize_e4m3_delayed
    assert f(FAKE, 0, 16, FAKE, None, FAKE, None) == hg.HGEMM_ERR_INVALID_VALUE   # no scale_in
    assert f(FAKE, 0, 16, FAKE, FAKE, None, None) == hg.HGEMM_ERR_INVALID_VALUE   # no amax_out
    assert f(None, 0, 16, FAKE, FAKE, FAKE, None) == hg.HGEMM_ERR_INVALID_VALUE
    assert f(FAKE, 3, 16, FAKE, FAKE, FAKE, None) == hg.HGEMM_ERR_INVALID_VALUE   # dtype
    assert f(FAKE + 4, 0, 16, FAKE, FAKE, FAKE, None) == hg.HGEMM_ERR_ALIGNMENT
    assert f(FAKE, 1, 16, FAKE + 8, FAKE, FAKE, None) == hg.HGEMM_ERR_ALIGNMENT
    assert f(FAKE, 0, 16, FAKE, FAKE + 2, FAKE, None) == hg.HGEMM_ERR_ALIGNMENT
    assert f(FAKE, 0, 16, FAKE, FAKE, FAKE + 1, None) == hg.HGEMM_ERR_ALIGNMENT


def test_debug_stall_hook_argument_checks():
    L = hg.lib()
    assert L.hgemm_debug_stalled_gemm(FAKE, FAKE, FAKE, 8, 8, 0, 0, None) == hg.HGEMM_ERR_INVALID_VALUE  # no K block
    assert L.hgemm_debug_stalled_gemm(FAKE, FAKE, FAKE, 8, 8, 16, 99, None) == hg.HGEMM_ERR_INVALID_VALUE
    assert L.hgemm_debug_stalled_gemm(FAKE, FAKE, FAKE, 8, 8, 24, 0, None) == hg.HGEMM_ERR_ALIGNMENT
