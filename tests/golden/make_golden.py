"""Generates tests/golden/oracle_small.npz: the oracle's outputs on small
seeded cases (BASELINE config-0 scene subset, random ellipses), committed so
that any change of the oracle's numerics is noticed by the CPU suite.

    python -m tests.golden.make_golden      # rewrites oracle_small.npz
"""

from __future__ import annotations

from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent / "oracle_small.npz"


def compute() -> dict:
    from jaxgs_b200.scene import config0_scene
    from oracle import oracle as O
    from tests.helpers import splats

    pool, cam, target = config0_scene()
    sel = np.arange(0, 4096, 8)
    small = {k: v[sel].copy() for k, v in pool.items()}
    proj = O.project_fwd(small, cam, degree=3, sh_dim=16)
    table = O.bin(proj, cam.width, cam.height, 16, 8, 1 << 15)
    fwd = O.raster_fwd(proj, table, cam.width, cam.height, 16, 8)
    img = fwd["rgb"].reshape(cam.height, cam.width, 3)
    loss, grad = O.loss(np.clip(img, 0, 1), target)
    rng = np.random.default_rng(7)
    ell = splats(rng, 256, 160, 96, radius=(0.5, 30.0), huge=2)
    etab = O.bin(ell, 160, 96, 16, 8, 1 << 14)
    return {
        "proj_mean": proj["mean"], "proj_conic": proj["conic"], "proj_color": proj["color"],
        "proj_visible": proj["visible"], "point_counts": table["point_counts"],
        "gaussian_ids": table["gaussian_ids"][:table["pair_count"]],
        "tile_offsets": table["tile_offsets"], "rgb": fwd["rgb"], "last": fwd["last"],
        "loss": np.float64(loss), "loss_grad": grad,
        "ellipse_counts": etab["point_counts"],
        "ellipse_ids": etab["gaussian_ids"][:etab["pair_count"]],
        "ellipse_offsets": etab["tile_offsets"],
    }


if __name__ == "__main__":
    np.savez_compressed(OUT, **compute())
    print(OUT)
