"""Generate ``tests/golden/golden.npz`` by running the reference's own Python code.

Run once, in a container where the reference checkout is available:

    python tests/golden/make_golden.py --reference <path to nibblegemm checkout>

It imports ``nibblegemm.quant`` from ``<reference>/python`` (the module whose
functions define the packed format and the CPU oracle, arvindcr4/nibblegemm
``python/nibblegemm/quant.py``) and records its outputs on seeded inputs.  The
fixtures are small (a few hundred KB) and are committed; nothing at test time
needs the reference checkout.

Cases (inputs are regenerated deterministically from the seeds in this file):

* ``pack_*``   -- ``pack_nibbles`` on the six involution shapes of the
  reference's ``tests/test_pack.py:45-52`` (seed ``K*31+N``).
* ``sweep_*``  -- ``dequantize`` on the exhaustive slot x value nibble sweep of
  ``tests/test_dequant.py:27-44`` with unit, 2**[-10, 10] and per-group 2**g
  scales, G in {64, 128}.
* ``quant_*``  -- ``quantize`` (RTN) of seeded ``N(0,1)*0.02`` weights, G in {64, 128}.
* ``clip_*``   -- ``quantize(clip_search=True)`` of seeded weights with planted
  outliers (so clipped candidates win in some groups), G in {64, 128}.
* ``mm_*``     -- ``reference_matmul`` on the BASELINE synthetic distribution
  (codes uniform 0..15, scales |N(0,1)|*0.02+1e-3, X ~ N(0,1)) at small shapes.
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

PACK_SHAPES = [(8, 1), (8, 4), (256, 64), (128, 130), (1024, 3), (2048, 1)]
MM_CASES = [  # (M, K, N, G, seed)
    (1, 256, 132, 128, 10),
    (3, 512, 256, 64, 11),
    (8, 1024, 96, 128, 12),
    (16, 256, 260, 128, 13),
    (17, 512, 128, 64, 14),
]


def sweep_nibbles(K: int, extra_cols: int, seed: int) -> np.ndarray:
    """Every (slot, value) pair isolated on a 0xF background, all-slots-equal
    columns, then random columns (the reference's dequant test pattern)."""
    k_off = np.arange(K) % 8
    slot, value = np.divmod(np.arange(128), 16)
    isolated = np.where(k_off[:, None] == slot[None, :], value[None, :], 15)
    uniform = np.tile(np.arange(16), (K, 1))
    rand = np.random.default_rng(seed).integers(0, 16, size=(K, extra_cols))
    return np.concatenate([isolated, uniform, rand], axis=1).astype(np.uint8)


def sweep_scales(kind: str, rows: int, N: int, seed: int) -> np.ndarray:
    if kind == "unit":
        return np.ones((rows, N), dtype=np.float32)
    if kind == "pow2":
        s = (2.0 ** np.random.default_rng(seed).uniform(-10.0, 10.0, size=(rows, N))).astype(np.float32)
        s[0, :4] = [2.0**-10, 2.0**10, 1.0, 2.0**-3]
        return s
    if kind == "group":
        return np.repeat((2.0 ** np.arange(rows, dtype=np.float32))[:, None], N, axis=1)
    raise ValueError(kind)


SWEEPS = [  # (name, K, extra_cols, nibble seed, scale kind, scale seed)
    ("unit", 128, 20, 0, "unit", 0),
    ("pow2", 256, 20, 1, "pow2", 2),
    ("group", 512, 4, 5, "group", 0),
]


def mm_inputs(M, K, N, G, seed):
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, 16, size=(K, N), dtype=np.uint8)
    scales = (np.abs(rng.standard_normal((K // G, N), dtype=np.float32)) * 0.02 + 1e-3).astype(np.float16)
    x = rng.standard_normal((M, K), dtype=np.float32).astype(np.float16)
    return codes, scales, x


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path to the nibblegemm checkout")
    ap.add_argument("--out", default=os.path.join(HERE, "golden.npz"))
    args = ap.parse_args()

    sys.dont_write_bytecode = True
    sys.path.insert(0, os.path.join(args.reference, "python"))
    import torch
    from nibblegemm import quant as ref  # the reference module itself

    out = {}
    for K, N in PACK_SHAPES:
        qu = np.random.default_rng(K * 31 + N).integers(0, 16, size=(K, N), dtype=np.uint8)
        out[f"pack_{K}x{N}"] = ref.pack_nibbles(qu)

    for name, K, extra, nseed, kind, sseed in SWEEPS:
        qu = sweep_nibbles(K, extra, nseed)
        for G in (64, 128):
            s = sweep_scales(kind, K // G, qu.shape[1], sseed)
            qw = ref.QuantizedWeight(
                qweight=torch.from_numpy(ref.pack_nibbles(qu)),
                scales=torch.from_numpy(s).to(torch.float16), group_size=G, K=K, N=qu.shape[1])
            out[f"sweep_{name}_g{G}_scales"] = qw.scales.numpy()
            out[f"sweep_{name}_g{G}_deq"] = ref.dequantize(qw).numpy()

    for G in (64, 128):
        g = torch.Generator().manual_seed(100 + G)
        W = torch.randn(256, 72, generator=g) * 0.02
        qw = ref.quantize(W, group_size=G)
        out[f"quant_g{G}_W"] = W.numpy()
        out[f"quant_g{G}_qweight"] = qw.qweight.numpy()
        out[f"quant_g{G}_scales"] = qw.scales.numpy()

    for G in (64, 128):
        g = torch.Generator().manual_seed(200 + G)
        W = torch.randn(512, 40, generator=g) * 0.02
        W[::37, ::3] *= 8.0  # outliers: the MSE search clips some groups
        qw = ref.quantize(W, group_size=G, clip_search=True)
        out[f"clip_g{G}_W"] = W.numpy()
        out[f"clip_g{G}_qweight"] = qw.qweight.numpy()
        out[f"clip_g{G}_scales"] = qw.scales.numpy()

    for M, K, N, G, seed in MM_CASES:
        codes, scales, x = mm_inputs(M, K, N, G, seed)
        qw = ref.QuantizedWeight(qweight=torch.from_numpy(ref.pack_nibbles(codes)),
                                 scales=torch.from_numpy(scales), group_size=G, K=K, N=N)
        y = ref.reference_matmul(torch.from_numpy(x), qw)
        out[f"mm_{M}x{K}x{N}_g{G}_s{seed}"] = y.numpy()

    np.savez_compressed(args.out, **out)
    print(f"wrote {len(out)} arrays to {args.out} ({os.path.getsize(args.out)} bytes)")


if __name__ == "__main__":
    main()
