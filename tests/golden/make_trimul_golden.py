"""Generate tests/golden/trimul_golden.npz: small seeded triangle-multiplication cases (outgoing and
incoming) with the float64 oracle's output (oracle/trimul_ref.py).

Shapes and masks follow the reference's own tri-mult tests (jackryan225/boltz-mlx): a ragged N with
20% of pairs masked (N = 45 there, tests/test_nax2_kernels.py:162-173; 33 here to keep the file small),
tiny N and B = 2, and a token-padding pair mask.  Values are synthetic (the reference's module dumps are
not available); inputs are rounded to fp16-representable values so they are stored losslessly; the
outputs are stored in float32 (relative rounding 6e-8, far below the 1e-5 fp32 bar).

    python tests/golden/make_trimul_golden.py
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle.trimul_ref import make_params, trimul_ref  # noqa: E402

OUT = Path(__file__).with_name("trimul_golden.npz")

CASES = [
    # name, B, N, mask kind, param set
    ("n1_b2", 2, 1, "rand", 0),
    ("n6_b2", 2, 6, "rand", 1),
    ("n17_pad", 1, 17, "pad", 0),
    ("n33_drop", 1, 33, "rand", 1),
    ("n9_nomask", 1, 9, "none", 0),
]


def mask_for(kind: str, B: int, N: int, g: torch.Generator):
    if kind == "none":
        return None
    if kind == "pad":
        tok = torch.ones(N)
        tok[-max(1, N // 5):] = 0.0
        return (tok[:, None] * tok[None, :]).expand(B, N, N).clone()
    return (torch.rand(B, N, N, generator=g) > 0.2).float()


def main():
    data = {}
    params = {0: make_params(200, ln_identity=True), 1: make_params(201)}
    for pid, p in params.items():
        for k, v in p.items():
            data[f"p{pid}_{k}"] = v.half().float().numpy()  # stored values are the ones used
    params = {pid: {k: torch.from_numpy(data[f"p{pid}_{k}"]) for k in p} for pid, p in params.items()}
    g = torch.Generator().manual_seed(7)
    for name, B, N, kind, pid in CASES:
        z = torch.randn(B, N, N, 128, generator=g).half().float()
        m = mask_for(kind, B, N, g)
        data[f"{name}_meta"] = np.array([B, N, pid], np.int64)
        data[f"{name}_z"] = z.half().numpy()
        if m is not None:
            data[f"{name}_mask"] = m.numpy().astype(np.uint8)
        for outgoing, tag in ((True, "out"), (False, "in")):
            y = trimul_ref(z.double(), None if m is None else m.double(), params[pid], outgoing=outgoing,
                           dtype=torch.float64)
            data[f"{name}_y_{tag}"] = y.numpy().astype(np.float32)
    np.savez_compressed(OUT, **data)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(CASES)} cases)")


if __name__ == "__main__":
    main()
