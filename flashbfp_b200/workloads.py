"""Seeded synthetic workloads for the OABF weight-streaming path.

No checkpoint or dataset is involved: the benchmark configurations are defined
by weight distributions and layer shapes, which these generators reproduce.

* ``config1_weight``: W[4096, 4096] fp32 ~ N(0, 0.02), 1.5% of entries at
  uniform random positions replaced by +-U(10, 50) * 0.02 (seed 0).
* ``decode_weight``: bf16 W ~ N(0, 0.02), 1.5% of entries at uniform random
  positions replaced by StudentT(df=3) * 20 * 0.02 (seed = base + layer id).
* ``GEMMA12B_LAYER``: the linear shapes (out N x in K) of one 12B-class decoder
  layer: hidden 3840, 16 query heads and 8 KV heads of 256, GeGLU MLP 15360.
* ``LLAMA70B_LAYER``: the same for the 70B-class stress layer: hidden 8192, 64 query heads
  and 8 KV heads of 128, MLP 28672.

Generators take a torch ``device`` so that large layers can be drawn directly
in device memory.
"""
from __future__ import annotations

import numpy as np
import torch

HIDDEN = 3840
GEMMA12B_LAYER = {
    # name: (N_out, K_in)
    "q_proj": (4096, 3840),
    "k_proj": (2048, 3840),
    "v_proj": (2048, 3840),
    "o_proj": (3840, 4096),
    "gate_proj": (15360, 3840),
    "up_proj": (15360, 3840),
    "down_proj": (3840, 15360),
}
# the 70B-class stress shapes: hidden 8192, 64 query / 8 KV heads of 128, MLP 28672
LLAMA70B_LAYER = {
    "q_proj": (8192, 8192),
    "k_proj": (1024, 8192),
    "v_proj": (1024, 8192),
    "o_proj": (8192, 8192),
    "gate_proj": (28672, 8192),
    "up_proj": (28672, 8192),
    "down_proj": (8192, 28672),
}
# fused launch groups used by decode: q|k|v and gate|up share their input
GEMMA12B_FUSED = {
    "qkv_proj": (8192, 3840),
    "o_proj": (3840, 4096),
    "gate_up_proj": (30720, 3840),
    "down_proj": (3840, 15360),
}


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def config1_weight(n: int = 4096, k: int = 4096, seed: int = 0, frac: float = 0.015,
                   device="cpu") -> torch.Tensor:
    g = _gen(seed, device)
    W = torch.randn(n, k, generator=g, device=device) * 0.02
    cnt = int(round(frac * n * k))
    pos = torch.randperm(n * k, generator=g, device=device)[:cnt]
    mag = torch.empty(cnt, device=device).uniform_(10.0, 50.0, generator=g) * 0.02
    sgn = torch.randint(0, 2, (cnt,), generator=g, device=device).float() * 2 - 1
    W.view(-1)[pos] = sgn * mag
    return W


def student_t(shape, df: int, g: torch.Generator, device="cpu") -> torch.Tensor:
    z = torch.randn(shape, generator=g, device=device)
    chi = torch.zeros(shape, device=device)
    for _ in range(df):
        chi += torch.randn(shape, generator=g, device=device) ** 2
    return z / torch.sqrt(chi / df)


def decode_weight(n: int, k: int, seed: int, frac: float = 0.015, scale: float = 20.0,
                  device="cpu", dtype=torch.bfloat16) -> torch.Tensor:
    g = _gen(seed, device)
    W = torch.randn(n, k, generator=g, device=device) * 0.02
    cnt = int(round(frac * n * k))
    if cnt:
        pos = torch.randperm(n * k, generator=g, device=device)[:cnt]
        W.view(-1)[pos] = student_t((cnt,), 3, g, device) * (scale * 0.02)
    return W.to(dtype)


def activations(m: int, k: int, seed: int, device="cpu", dtype=torch.bfloat16) -> torch.Tensor:
    g = _gen(seed, device)
    return torch.randn(m, k, generator=g, device=device).to(dtype)


# ----------------------------------------------------------------------------
# small cases with crafted edge blocks (golden fixtures)
# ----------------------------------------------------------------------------

def edge_matrix(dt: str) -> torch.Tensor:
    """64 x 80 matrix whose blocks hit the packing edge cases: all-zero
    blocks, maxima just below a power of two (the log2 rounding codes),
    negative values that quantise to mantissa 0 (-0.0 on dequant), a negative
    16th element (int16 sign wrap), mantissa 15 in nibble 7 and 15 (int32
    wrap), block maxima in [1e-8, 1e-7) and below 1e-8, exact half-way
    mantissas, values exactly at and just above the clamped threshold 0.20,
    and a ragged K (80 = 5 blocks) with N=64."""
    rng = np.random.default_rng(1234)
    W = (rng.standard_normal((64, 80)) * 0.02).astype(np.float32)
    f32 = np.float32

    def below_pow2(e, j):  # x = 2^(e+1) * (1 - j * 2^-24) as fp32 (or bf16 code for dt=bf16)
        if dt == "bf16":
            code = ((e + 127) << 7) | (127 - (j - 1))
            return (np.array([code << 16], dtype=np.uint32).view(np.float32))[0]
        code = ((e + 127) << 23) | ((1 << 23) - j)
        return np.array([code], dtype=np.uint32).view(np.float32)[0]

    r = 0
    W[r, 0:16] = 0.0                                          # all-zero block
    W[r, 16:32] = rng.standard_normal(16).astype(f32) * 1e-9  # bmax < 1e-8
    W[r, 32:48] = np.linspace(-9e-8, 9e-8, 16).astype(f32)    # bmax in [1e-8, 1e-7)
    W[r, 48:64] = -np.abs(W[r, 48:64])                        # all negative
    r += 1
    for e, js in ((-17, (10, 11, 12)), (-16, (4, 5, 6)), (-9, (5, 6)), (-8, (1, 2, 3)),
                  (-5, (2, 3)), (-4, (1, 2)), (-3, (1, 2))):
        for j in js:
            blk = (rng.standard_normal(16) * 0.3).astype(f32) * below_pow2(e, j)
            blk[int(rng.integers(16))] = below_pow2(e, j)
            W[r, (j % 5) * 16:(j % 5) * 16 + 16] = np.clip(blk, -0.19, 0.19)
        r += 1
    blk = np.full(16, 1e-4, dtype=f32)
    blk[0] = 0.05
    blk[1:8] = -1e-4                                          # -> m = 0 with sign = 1
    blk[15] = -0.01                                           # sign bit 15
    W[r, 0:16] = blk
    blk = np.full(16, 0.001, dtype=f32)
    blk[7] = 0.06
    blk[15] = 0.06                                            # nibble 7 of both words = 15
    W[r, 16:32] = blk
    blk = np.zeros(16, dtype=f32)
    blk[0] = 2.0 ** -5
    blk[1] = 2.0 ** -6                                        # aligned 0.5 -> 7.5 -> 8 (half-even)
    blk[2] = -(2.0 ** -6)
    blk[3] = 3 * 2.0 ** -7
    W[r, 32:48] = blk
    W[r, 48] = 0.2                                            # exactly at clamped threshold
    W[r, 49] = np.nextafter(f32(0.2), f32(1.0))               # just above (fp32)
    W[r, 50] = 0.20019531                                     # bf16(0.2) neighbourhood
    W[r, 51] = 0.2003
    W[r, 64:80] = -0.0
    r += 1
    # outliers so the threshold clamps to 0.20
    pos = rng.choice(np.arange(r * 80, 64 * 80), size=120, replace=False)
    W.reshape(-1)[pos] = (rng.uniform(10, 50, size=120) * 0.02 *
                          rng.choice([-1.0, 1.0], size=120)).astype(f32)
    t = torch.from_numpy(W)
    return t.to(torch.bfloat16) if dt == "bf16" else t


def golden_cases():
    """name -> (W, [X...], bias_seed or None). Small enough for fixtures."""
    cases = {}
    W = config1_weight(128, 192, seed=0)
    cases["cfg1_small_fp32"] = (W, [activations(1, 192, 1, dtype=torch.float32),
                                    activations(16, 192, 2, dtype=torch.float32)], None)
    W = decode_weight(192, 256, seed=7)
    cases["decode_t3_bf16"] = (W, [activations(m, 256, 10 + m) for m in (1, 4, 16)], 3)
    g = _gen(11, "cpu")
    cases["gauss_bf16"] = ((torch.randn(128, 128, generator=g) * 0.02).to(torch.bfloat16),
                           [activations(2, 128, 12)], None)
    cases["gauss_pad_fp32"] = (torch.randn(100, 70, generator=g) * 0.05,
                               [activations(3, 70, 13, dtype=torch.float32)], 5)
    W = decode_weight(65, 33, seed=14, frac=0.03)
    cases["pad_t3_bf16"] = (W, [activations(5, 33, 15)], None)
    cases["edge_fp32"] = (edge_matrix("fp32"), [activations(4, 80, 16, dtype=torch.float32)], None)
    cases["edge_bf16"] = (edge_matrix("bf16"), [activations(4, 80, 17)], 6)
    cases["tiny_1x1_fp32"] = (torch.tensor([[0.3]]), [activations(1, 1, 18, dtype=torch.float32)], None)
    cases["tiny_1x16_bf16"] = ((torch.randn(1, 16, generator=g) * 0.1).to(torch.bfloat16),
                               [activations(1, 16, 19)], None)
    cases["tiny_2x3_fp32"] = (torch.randn(2, 3, generator=g) * 0.1,
                              [activations(2, 3, 20, dtype=torch.float32)], None)
    return cases


def fullsize_cases():
    """Full-size matrices whose packed-byte digests are pinned by fixtures."""
    return {
        "config1_4096x4096_fp32": config1_weight(4096, 4096, seed=0),
        "decode_t3_3840x2048_bf16": decode_weight(2048, 3840, seed=100),
    }
