"""Shared test inputs: the reference's LCG vectors and seeded synthetic rows."""
import numpy as np

# Type ids (reference gguf.rs:36-83).
F32, F16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0 = 0, 1, 2, 3, 6, 7, 8
Q2_K, Q3_K, Q4_K, Q5_K, Q6_K = 10, 11, 12, 13, 14
IQ2_XXS, IQ2_XS, IQ3_XXS, IQ4_NL, IQ3_S, IQ2_S, IQ4_XS, BF16 = 16, 17, 18, 20, 21, 22, 23, 30

NAMES = {F32: "F32", F16: "F16", Q4_0: "Q4_0", Q4_1: "Q4_1", Q5_0: "Q5_0", Q5_1: "Q5_1", Q8_0: "Q8_0",
         Q2_K: "Q2_K", Q3_K: "Q3_K", Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K", IQ2_XXS: "IQ2_XXS", IQ2_XS: "IQ2_XS", IQ3_XXS: "IQ3_XXS",
         IQ4_NL: "IQ4_NL", IQ3_S: "IQ3_S", IQ2_S: "IQ2_S", IQ4_XS: "IQ4_XS", BF16: "BF16"}
KQUANT = [Q8_0, Q6_K, Q4_K, Q5_K, Q4_0, Q4_1, Q5_0, Q5_1]
LEGACY = [Q4_0, Q4_1, Q5_0, Q5_1]
IQ = [IQ2_XXS, IQ2_XS, IQ2_S, IQ3_XXS, IQ3_S, IQ4_NL, IQ4_XS]
PLAIN = [F32, F16, BF16]
# K-quants beyond the reference's type set (ggml block layouts)
KQUANT_EXTRA = [Q2_K, Q3_K]


def lcg_vec(n, seed=0x12345678):
    """quant.rs:636-645 test_vec / quant_iq.rs:1195-1203 (wrapping LCG, f32 math)."""
    s = seed
    out = np.empty(n, dtype=np.float32)
    umax = np.float32(4294967295.0)
    for i in range(n):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = (np.float32(s) / umax - np.float32(0.5)) * np.float32(4.0)
    return out


def f32_to_bf16_bits(x):
    """f32 -> BF16 bits, round to nearest even (NaN kept quiet)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(b):
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def sweep_rows(n_rows, ne0, seed):
    """Encoder-sweep distribution: N(0, 0.02) with 0.1% outliers at +-8 sigma,
    per-column log-normal imatrix (sigma 1.5). Returns (bf16 bits, imatrix)."""
    rng = np.random.default_rng(seed)
    w = rng.normal(0.0, 0.02, size=(n_rows, ne0)).astype(np.float32)
    k = max(1, int(round(w.size * 0.001)))
    idx = rng.choice(w.size, size=k, replace=False)
    w.reshape(-1)[idx] = rng.choice(np.array([-0.16, 0.16], dtype=np.float32), size=k)
    im = np.exp(rng.normal(0.0, 1.5, size=ne0)).astype(np.float32)
    return f32_to_bf16_bits(w), im


def student_rows(n_rows, ne0, seed, nu=5.0):
    """IQ distribution: Student-t(5) scaled to std 0.02, imatrix log-normal (sigma 1)."""
    rng = np.random.default_rng(seed)
    w = (rng.standard_t(nu, size=(n_rows, ne0)) * (0.02 / np.sqrt(nu / (nu - 2.0)))).astype(np.float32)
    im = np.exp(rng.normal(0.0, 1.0, size=ne0)).astype(np.float32)
    return f32_to_bf16_bits(w), im


def edge_rows(ne0):
    """Rows that exercise the reference's degenerate branches."""
    rows = []
    rows.append(np.zeros(ne0, np.float32))                              # all zero
    rows.append(np.full(ne0, 0.0123, np.float32))                        # constant positive
    rows.append(np.full(ne0, -0.5, np.float32))                          # constant negative
    r = np.zeros(ne0, np.float32); r[7] = 1.0; rows.append(r)            # single outlier
    r = np.zeros(ne0, np.float32); r[::2] = -0.0; r[1::3] = 3e-39; rows.append(r)  # -0 and denormals
    r = np.linspace(-1, 1, ne0, dtype=np.float32); rows.append(r)        # ramp
    r = np.where(np.arange(ne0) % 32 < 16, 1e-20, -2.5).astype(np.float32); rows.append(r)  # tiny vs big
    r = np.full(ne0, 1e-16, np.float32); rows.append(r)                  # below GROUP_MAX_EPS
    r = (np.arange(ne0) % 7 - 3).astype(np.float32) * 0.25; rows.append(r)  # exact .5 ties after scaling
    return np.stack(rows)
