"""BASELINE.json problem shapes as oracle ``ConvCase`` objects (test infra).

Each entry: (name, case, input_std, precisions).  Inputs are seeded synthetic
data with the shapes and distributions the configs state: input parts iid
N(0, std^2) with std 1 (0.1 for the MRI layer), weights U(+-1/sqrt(C*R*S)).
"""

from .oracle import ConvCase

# the reference's CPU-runnable case.
CPU_CASE = ConvCase(1, 32, 32, 32, 32, 3, 3, 1, 1, 1, 1)

BASELINE_CASES = [
    # batch-1 3x3 s1 p1 sweep (single GPU), forward and forward_planar.
    ("b1_32_64_56", ConvCase(1, 32, 56, 56, 64, 3, 3, 1, 1, 1, 1), 1.0, ("tf32",)),
    ("b1_64_128_28", ConvCase(1, 64, 28, 28, 128, 3, 3, 1, 1, 1, 1), 1.0, ("tf32",)),
    ("b1_128_256_14", ConvCase(1, 128, 14, 14, 256, 3, 3, 1, 1, 1, 1), 1.0, ("tf32",)),
    ("b1_256_512_7", ConvCase(1, 256, 7, 7, 512, 3, 3, 1, 1, 1, 1), 1.0, ("tf32",)),
    # batched compute-bound layer.
    ("b64_128_128_56", ConvCase(64, 128, 56, 56, 128, 3, 3, 1, 1, 1, 1), 1.0, ("tf32",)),
    # stride-2 and pointwise variants.
    ("b32_s2_64_128_112", ConvCase(32, 64, 112, 112, 128, 3, 3, 2, 2, 1, 1), 1.0, ("tf32",)),
    ("b32_1x1_256_1024_28", ConvCase(32, 256, 28, 28, 1024, 1, 1, 1, 1, 0, 0), 1.0, ("tf32",)),
    # MRI-style large image, TF32 and 3xTF32.
    ("b32_64_64_320", ConvCase(32, 64, 320, 320, 64, 3, 3, 1, 1, 1, 1), 0.1, ("tf32", "3xtf32")),
]
