"""Generate tests/golden/reference_outputs.npz from the reference's own kernels.

Runs on a B200: loads oracle/_ref/libmfa_ref.so (the unmodified reference CuTe and WMMA
kernels compiled from their sources by oracle/build_ref.py) and records their fp16 outputs
for seeded inputs. Inputs are NOT stored: they are regenerated bit-identically from
`make_inputs` (numpy PCG64, seed per case); a sha256 of the input bytes is stored to detect
drift.

Cases: the three shapes of the reference test (tests/test_forward.py:9-18: (1,2,128,64),
(2,1,256,64), (1,2,2048,64), N(0,1) inputs) for both kernels, plus two stress cases shaped
like the long-sequence config (q,k ~ N(0,3^2): peaky softmax) and the short-sequence config
(uniform[-1,1]) at sizes the oracle finishes in seconds.

Usage (GPU box): python tests/golden/make_golden.py [--out PATH]
(then copy the file to tests/golden/reference_outputs.npz and commit it with this script).
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
OUT = Path(__file__).resolve().parent / "reference_outputs.npz"

# name -> (shape, distribution, seed, kernels)
CASES = {
    "ref_b1h2n128": ((1, 2, 128, 64), "normal", 0, ("cute", "wmma")),
    "ref_b2h1n256": ((2, 1, 256, 64), "normal", 1, ("cute", "wmma")),
    "ref_b1h2n2048": ((1, 2, 2048, 64), "normal", 2, ("cute",)),
    "peaky_b1h2n512": ((1, 2, 512, 64), "peaky", 3, ("cute",)),
    "uniform_b4h1n256": ((4, 1, 256, 64), "uniform", 4, ("cute",)),
}


def make_inputs(shape, dist: str, seed: int):
    """fp16 q, k, v for a case; identical on every machine (numpy PCG64)."""
    rng = np.random.default_rng(seed)
    if dist == "normal":
        q, k, v = (rng.standard_normal(shape, dtype=np.float32) for _ in range(3))
    elif dist == "peaky":
        q = 3.0 * rng.standard_normal(shape, dtype=np.float32)
        k = 3.0 * rng.standard_normal(shape, dtype=np.float32)
        v = rng.standard_normal(shape, dtype=np.float32)
    elif dist == "uniform":
        q, k, v = (rng.random(shape, dtype=np.float32) * 2.0 - 1.0 for _ in range(3))
    else:
        raise ValueError(dist)
    return tuple(x.astype(np.float16) for x in (q, k, v))


def input_digest(q, k, v) -> str:
    h = hashlib.sha256()
    for x in (q, k, v):
        h.update(np.ascontiguousarray(x).tobytes())
    return h.hexdigest()


def main() -> None:
    import argparse

    ap = argparse.ArgumentParser()
    ap.add_argument("--out", type=Path, default=OUT)
    out_path = ap.parse_args().out
    sys.path.insert(0, str(ROOT))
    import torch

    from oracle import ref

    if not ref.available():
        raise SystemExit("oracle/_ref/libmfa_ref.so missing: run python oracle/build_ref.py")
    arrays = {}
    for name, (shape, dist, seed, kernels) in CASES.items():
        q, k, v = make_inputs(shape, dist, seed)
        arrays[f"{name}__digest"] = np.array(input_digest(q, k, v))
        tq, tk, tv = (torch.from_numpy(x).cuda() for x in (q, k, v))
        for kern in kernels:
            out = ref.reference_forward(tq, tk, tv, kernel=kern)
            torch.cuda.synchronize()
            arrays[f"{name}__{kern}"] = out.cpu().numpy()
            print(name, kern, float(out.float().abs().max()))
    np.savez_compressed(out_path, **arrays)
    print("wrote", out_path)


if __name__ == "__main__":
    main()
