"""The reference's known-answer tests for the CPU ops, restated as data.

Each case reproduces the inputs and expected values of one test in
tests/src/cpu_ops/*.cpp of dsuarez01/minfer (file:line given per case), with
the tolerance that test uses. `run_*` functions take an op backend (the
oracle restatement, the reference's own compiled ops, or the CUDA ops) so the
same cases pin every implementation.
"""
from __future__ import annotations

import math

import numpy as np

f32 = np.float32


def _bf16(bits: int, n: int) -> np.ndarray:
    return np.full(n, bits, dtype=np.uint16)


# ------------------------------------------------------------------ matmul
# tests/src/cpu_ops/test_matmul.cpp
def matmul_cases():
    cases = []
    inp16 = np.arange(1, 17, dtype=f32)
    w = np.zeros((16, 16), f32)
    np.fill_diagonal(w, 1.0)
    cases.append(("identity", inp16, w.ravel(), 0, 16, 16, inp16.copy(), 1e-6))  # :11-33
    w = np.ones((16, 16), f32)
    w[2, :] = -2.0
    exp = np.full(16, 136.0, f32)
    exp[2] = -272.0
    cases.append(("square", inp16, w.ravel(), 0, 16, 16, exp, 1e-6))  # :35-62
    inp32 = np.array([1, 2, -3, -4, 0.5, 1.5, -0.5, 2.5, 0.1, 0.2, 0.3, 0.4, -0.1, -0.2, -0.3, -0.4,
                      1, 1, 1, 1, 2, 2, 2, 2, -1, -1, -1, -1, -2, -2, -2, -2], f32)
    pat = np.array([1.0, -0.5, 2.0, 0.25], f32)
    w = np.tile(np.tile(pat, 8), (16, 1)).astype(f32)
    exp = np.zeros(16, f32)
    for i in range(16):  # sequential fp32 accumulation as in the test (:87-94)
        acc = f32(0)
        for j in range(32):
            acc = f32(acc + f32(inp32[j] * w[i, j]))
        exp[i] = acc
    cases.append(("rectangular", inp32, w.ravel(), 0, 16, 32, exp, 1e-6))  # :64-99
    cases.append(("zero_matrix", np.arange(1, 33, dtype=f32), np.zeros(512, f32), 0, 16, 32, np.zeros(16, f32),
                  1e-6))  # :101-121
    cases.append(("zero_vector", np.zeros(16, f32), np.arange(1, 257, dtype=f32), 0, 16, 16, np.zeros(16, f32),
                  1e-6))  # :123-142
    big = np.array([1000, -2000, 500, -1500, 100, 200, -300, 400, 50, -75, 25, -125, 10, 20, -30, 40], f32)
    w = np.tile(np.array([0.001, -0.001] * 8, f32), (16, 1))
    exp = np.zeros(16, f32)
    for i in range(16):
        acc = f32(0)
        for j in range(16):
            acc = f32(acc + f32(big[j] * w[i, j]))
        exp[i] = acc
    cases.append(("large_values", big, w.ravel(), 0, 16, 16, exp, 1e-3))  # :144-175
    return cases


def matmul_16bit_cases():
    # (name, dtype code, weight bits, input, offset, d_out, d_in, expected, tol)
    ones = np.ones(32, f32)
    return [
        ("fp16", 1, np.full(512, 0x3800, np.uint16), ones, 0, 16, 32, np.full(16, 16.0, f32), 1e-3),  # :177-199
        ("bf16", 2, np.full(512, 0x3F00, np.uint16), ones, 0, 16, 32, np.full(16, 16.0, f32), 1e-3),  # :201-223
    ]


def offset_case():
    """test_offset (:225-271): expert 2 of a [4, 8, 16] tensor in f32/f16/bf16."""
    n_exp, d_out, d_in, e = 4, 8, 16, 2
    x = np.arange(1, 17, dtype=f32)
    sign = np.array([1.0 if (i // (d_out * d_in)) % 2 == 0 else -1.0 for i in range(512)], f32)
    w16 = np.where(sign > 0, 0x3C00, 0xBC00).astype(np.uint16)
    wbf = np.where(sign > 0, 0x3F80, 0xBF80).astype(np.uint16)
    return x, sign, w16, wbf, e * d_out * d_in, d_out, d_in


# ------------------------------------------------------------------ rmsnorm
# tests/src/cpu_ops/test_rmsnorm.cpp
def rmsnorm_cases():
    eps = 1e-6
    out = []
    rms = math.sqrt(f32(25.0 / 4.0 + eps))
    out.append(("unit_vector", np.array([3, 4, 0, 0], f32), np.ones(4, f32), eps,
                np.array([3 / rms, 4 / rms, 0, 0], f32), 1e-6))  # :10-25
    rms = math.sqrt(f32(14.0 / 3.0 + eps))
    out.append(("scaling", np.array([1, 2, 3], f32), np.array([2, 0.5, 1], f32), eps,
                np.array([1 / rms * 2, 2 / rms * 0.5, 3 / rms], f32), 1e-6))  # :27-41
    out.append(("zero_input", np.zeros(3, f32), np.ones(3, f32), eps, np.zeros(3, f32), 1e-6))  # :43-55
    rms = math.sqrt(f32(16.0 / 4 + eps))
    out.append(("uniform", np.full(4, 2, f32), np.ones(4, f32), eps, np.full(4, 2 / rms, f32), 1e-6))  # :57-69
    return out


# ------------------------------------------------------------------ rope
# tests/src/cpu_ops/test_rope.cpp (base 10000)
def rope_cases():
    c1, s1 = math.cos(1.0), math.sin(1.0)
    c01, s01 = math.cos(0.01), math.sin(0.01)
    return [
        # (name, neox, input, d_head, d_rot, pos, expected or None, tol)
        ("il_pos0", False, np.array([1, 2, 3, 4], f32), 4, 4, 0, np.array([1, 2, 3, 4], f32), 1e-6),  # :8-23
        ("il_single", False, np.array([1, 0, 0, 1], f32), 4, 4, 1, np.array([c1, s1, -s01, c01], f32), 1e-6),
        ("neox_pos0", True, np.array([1, 2, 3, 4], f32), 4, 4, 0, np.array([1, 2, 3, 4], f32), 1e-6),  # :68-83
        ("neox_single", True, np.array([1, 0, 0, 1], f32), 4, 4, 1, np.array([c1, -s01, s1, c01], f32),
         1e-6),  # :85-106
    ]


def rope_partial_cases():
    # partial rotary (:48-66, :108-126): dims past d_rot keep the output buffer's value
    return [("il_partial", False), ("neox_partial", True)]


# ------------------------------------------------------------------ attention
# tests/src/cpu_ops/test_attn.cpp
def attn_weights_case():
    """test_attention_weights (:86-119)."""
    q = np.ones(3, f32)
    k = np.array([1, 1, 1, -1, -1, -1], f32)
    v = np.array([1, 0, 0, 0, 1, 0], f32)
    a = f32(1 / math.sqrt(3) * 3)
    e1, e2 = math.exp(a), math.exp(-a)
    w = np.array([e1 / (e1 + e2), e2 / (e1 + e2)], f32)
    return q, k, v, 2, 3, 3, w, np.array([w[0], w[1], 0], f32), 1e-6


# ------------------------------------------------------------------ route
# tests/src/cpu_ops/test_route.cpp
def route_cases():
    cases = []
    x = np.array([1, 2, 3, 1, 2, 3, 1, 2, 3, 1, 2, 3, 1, 2, 3, 1], f32)
    w = np.zeros((4, 16), f32)
    for i in range(4):
        for j in range(16):
            w[i, j] = 1.0 if (i == 3 or i == j % 3) else 0.0
    cases.append(("single_expert", x, w, 4, 1, [3], None))  # :9-39
    w = np.repeat(np.array([2, 4, 1, 6, 3], f32)[:, None], 16, axis=1)
    cases.append(("top_k_selection", np.ones(16, f32), w, 5, 3, [3, 1, 4], None))  # :41-70
    x = np.zeros(16, f32)
    x[0] = 1
    w = np.zeros((3, 16), f32)
    w[:, 0] = [10, 5, 1]
    cases.append(("score_normalization", x, w, 3, 2, [0, 1], "normalised"))  # :72-102
    w = np.zeros((4, 16), f32)
    w[:, 0] = [2, 4, 1, 3]
    cases.append(("expert_ordering", x, w, 4, 4, [1, 3, 0, 2], "descending"))  # :104-137
    return cases


# ------------------------------------------------------------------ softmax / silu
# tests/src/cpu_ops/test_softmax.cpp, test_silu.cpp
def softmax_cases():
    return [
        ("uniform", np.zeros(3, f32), np.full(3, 1 / 3, f32), 1e-6),  # :8-17
        ("one_hot", np.array([-1e6, 0, -1e6, -1e6], f32), np.array([0, 1, 0, 0], f32), 1e-6),  # :19-28
    ]


def silu_cases():
    return [(x, x / (1 + math.exp(-x)), 1e-6) for x in (0.0, 1.0, 2.0, -1.0, -2.0)]  # :8-43
