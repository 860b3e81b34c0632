"""Regenerate ``harmonic_basis_v1.json`` from an ICTC-O3 source tree.

The ICTC angular basis for each degree l is a (Dsym(l), 2l+1) float64 matrix
that maps harmonic coordinates to monomial coefficients.  It is a *frozen*
choice inside a degenerate nullspace, so it cannot be recomputed from the
mathematics alone: every released checkpoint, CG tensor and direction
harmonic depends on the exact columns.  The reference ships it as
``ictc_o3/basis/_ictd_basis/v1/harmonic_basis_l{l}.pt`` and pins each
tensor's bytes with SHA-256 (``ictc_o3/basis/ictd_irreps.py:633-693``).

This script copies those tensors (l = 0..LMAX) into a text table, storing each
value with ``float.hex`` so the round trip is exact, and re-checks the pinned
digest of every tensor.  Usage::

    python make_basis_table.py <path-to-ictc_o3-source-root> [LMAX]
"""
import hashlib
import json
import os
import sys

import numpy as np


def main(argv):
    root = argv[1]
    lmax = int(argv[2]) if len(argv) > 2 else 6
    import torch
    from harmonic_basis_pins import BASIS_SHA256  # noqa: E402  (same folder)
    table = {"format": "ictd-canonical-harmonic-basis", "version": "v1", "degrees": {}}
    for l in range(lmax + 1):
        path = os.path.join(root, "ictc_o3", "basis", "_ictd_basis", "v1", f"harmonic_basis_l{l}.pt")
        blob = torch.load(path, map_location="cpu", weights_only=True)
        tensor = blob["tensor"].detach().to(torch.float64).contiguous().numpy()
        digest = hashlib.sha256(np.ascontiguousarray(tensor).tobytes()).hexdigest()
        if digest != BASIS_SHA256[l]:
            raise SystemExit(f"digest mismatch for l={l}")
        table["degrees"][str(l)] = {
            "shape": list(tensor.shape),
            "sha256": digest,
            "values": [float(v).hex() for v in tensor.reshape(-1)],
        }
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "harmonic_basis_v1.json")
    with open(out, "w") as handle:
        json.dump(table, handle, indent=0)
    print("wrote", out)


if __name__ == "__main__":
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    main(sys.argv)
