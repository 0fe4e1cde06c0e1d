"""Generate tests/golden/triattn_golden.npz: small seeded triangle-attention cases with the float64
oracle's output (oracle/triattn_ref.py, fp32 rounding of masked logits kept).

The cases re-create the SHAPES and MASK PATTERNS of the reference's own tri-attention tests
(jackryan225/boltz-mlx): tiny / ragged N in {1, 2, 9, 17, 33} with B = 2 (tests/test_triatt_mma.py:42-51),
a fully masked query row and a masked key column (tests/test_triatt_mma.py:16-21), a ragged
token-padding pair mask with 10% of pair entries dropped (tests/test_trunk_vs_torch.py:84-103), and
both orientations (start / end node).  Values are synthetic (the reference's parity dumps are not
available); inputs are rounded to fp16-representable values so they are stored losslessly.

    python tests/golden/make_golden.py
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle.triattn_ref import make_params, tri_attention_ref  # noqa: E402

OUT = Path(__file__).with_name("triattn_golden.npz")

CASES = [
    # name, B, N, mask kind, param set
    ("n1_b2", 2, 1, "rand", 0),
    ("n2_b2", 2, 2, "rand", 1),
    ("n9_b2", 2, 9, "rows_cols", 0),
    ("n17_b1", 1, 17, "pad_drop", 1),
    ("n33_b1", 1, 33, "rows_cols", 0),
    ("n17_nomask", 1, 17, "none", 1),
]


def mask_for(kind: str, B: int, N: int, g: torch.Generator):
    if kind == "none":
        return None
    m = (torch.rand(B, N, N, generator=g) > 0.3).float()
    if kind == "rows_cols" and N > 7:
        m[:, 3, :] = 0.0  # fully masked query row
        m[:, :, 5] = 0.0  # one masked key column
        m[:, 7, :] = 0.0
    if kind == "pad_drop":
        tok = torch.ones(N)
        tok[-max(1, N // 5):] = 0.0  # ~20% padded tokens
        m = (tok[:, None] * tok[None, :]).expand(B, N, N).clone()
        m = m * (torch.rand(B, N, N, generator=g) > 0.1).float()
    return m


def main():
    data = {}
    params = {0: make_params(100, gate_bias=1.0, ln_identity=True), 1: make_params(101, gate_bias=None, ln_identity=False)}
    for pid, p in params.items():
        for k, v in p.items():
            if v is not None:
                data[f"p{pid}_{k}"] = v.numpy().astype(np.float32)
    for name, B, N, kind, pid in CASES:
        g = torch.Generator().manual_seed(sum(map(ord, name)))
        z = torch.randn(B, N, N, 128, generator=g).half().float()
        m = mask_for(kind, B, N, g)
        data[f"{name}_z"] = z.numpy().astype(np.float16)
        if m is not None:
            data[f"{name}_mask"] = m.numpy().astype(np.uint8)  # 0/1 masks
        data[f"{name}_meta"] = np.array([B, N, pid], np.int64)
        for starting in (True, False):
            y = tri_attention_ref(z, m, params[pid], starting=starting, dtype=torch.float64)
            data[f"{name}_y_{'start' if starting else 'end'}"] = y.numpy().astype(np.float32)
    np.savez_compressed(OUT, **data)
    print(OUT, OUT.stat().st_size, "bytes")


if __name__ == "__main__":
    main()
