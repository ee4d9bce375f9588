"""Shared helpers for the GPU parity tests: seeded inputs from the oracle's generator
(the same bytes go to the GPU and to the CPU oracle), a run through the C ABI, and a
check against the oracle under |c - ref| <= 1e-2*|ref| + 1e-3."""
from __future__ import annotations

import hashlib

import numpy as np
import torch

import oracle


def make_inputs(M: int, N: int, K: int, seed_a: int = 0, seed_b: int = 1, mean_a: float = 0.0, std_a: float = 1.0,
                mean_b: float = 0.0, std_b: float = 1.0, scaled: bool = True):
    """e4m3 A (MxK), B (NxK) and their scales, benchmark-config style (amax/448 per tensor) or,
    with scaled=False, the reference's raw cast of utils.hpp:27-33 (scale 1)."""
    if scaled:
        A, sa = oracle.make_quantized((M, K), seed_a, mean_a, std_a)
        B, sb = oracle.make_quantized((N, K), seed_b, mean_b, std_b)
    else:
        A = oracle.init_random_fp8(M * K, seed_a, mean_a, std_a).reshape(M, K)
        B = oracle.init_random_fp8(N * K, seed_b, mean_b, std_b).reshape(N, K)
        sa = sb = 1.0
    return A, B, sa, sb


def sha256(buf) -> str:
    """SHA-256 of a host array's or a device tensor's bytes (a device tensor is read back)."""
    if isinstance(buf, torch.Tensor):
        buf = buf.detach().contiguous().cpu().numpy()
    return hashlib.sha256(np.ascontiguousarray(buf).tobytes()).hexdigest()


def to_device(A: np.ndarray, B: np.ndarray, sa: float | None, sb: float | None, device="cuda:0"):
    """A, B and the scales on the device.  The e4m3 bytes the GPU will read are read back and
    hashed against the host buffers the oracle reads, so every parity test also proves that
    both sides computed from bit-identical inputs."""
    a = torch.from_numpy(A).to(device)
    b = torch.from_numpy(B).to(device)
    assert sha256(a) == sha256(A) and sha256(b) == sha256(B), "device operands differ from the oracle's bytes"
    ta = None if sa is None else torch.tensor([sa], dtype=torch.float32, device=device)
    tb = None if sb is None else torch.tensor([sb], dtype=torch.float32, device=device)
    return a, b, ta, tb


def c_bits(c: torch.Tensor) -> np.ndarray:
    return c.view(torch.int16).cpu().numpy().view(np.uint16)


def sample_rows(M: int, n: int, seed: int = 123) -> np.ndarray:
    """First, last, tile-edge and random rows (sorted, unique)."""
    rng = np.random.default_rng(seed)
    edge = [0, 1, 127, 128, 255, 256, M // 2, M - 129, M - 128, M - 2, M - 1]
    rows = set(r for r in edge if 0 <= r < M)
    rows.update(int(r) for r in rng.integers(0, M, size=max(0, n - len(rows))))
    return np.array(sorted(rows), dtype=np.int32)


def check_against_oracle(C_gpu: np.ndarray, A, B, sa: float, sb: float, rows=None):
    """Returns (mismatches, checked elements, first bad index)."""
    if rows is None:
        ref = oracle.gemm(A, B, sa, sb)
        got = C_gpu
    else:
        ref = oracle.gemm_rows(A, B, rows, sa, sb)
        got = np.ascontiguousarray(C_gpu[rows])
    bad, first = oracle.validate(got, ref)
    return bad, ref.size, first
