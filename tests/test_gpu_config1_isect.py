"""Tile intersection at BASELINE config 1 (1M Gaussians, one 1297x840 camera):
the tile ids, the depth order (ties by splat index), the splat ids of every
intersection and the per-tile offsets that ``rasterization()`` produces, bit for
bit against the CPU oracle's AccuTile sweep + stable sort + offset encode on the
same projected splats. At this size the tile buckets reach every sort path of
the library: the on-chip sort classes and, for the largest buckets, the global
radix fallback -- the size classes the small-scene tests build by hand."""

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests import _data
from tests._compare import as_np, assert_equal

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


@pytest.mark.parametrize("packed", [True, False])
def test_config1_intersections_bit_exact_vs_oracle(packed):
    import gsplat_b200

    d = _data.to(_data.config1(), DEV)
    W, H = d["width"], d["height"]
    with torch.no_grad():
        _, _, meta = gsplat_b200.rasterization(d["means"], d["quats"], d["scales"], d["opacities"],
                                               d["sh"], d["viewmats"], d["Ks"], W, H, sh_degree=3,
                                               far_plane=100.0, packed=packed)
    ts, tw, th = meta["tile_size"], meta["tile_width"], meta["tile_height"]
    keys = meta["isect_ids"]
    assert keys.numel() > 3_000_000
    if packed:
        image_ids = as_np(meta["camera_ids"])
        etpg, ekeys, eids = O.isect_tiles(as_np(meta["means2d"]), as_np(meta["radii"]),
                                          as_np(meta["depths"]), ts, tw, th, conics=as_np(meta["conics"]),
                                          opacities=as_np(meta["opacities"]), image_ids=image_ids,
                                          n_images=1)
    else:
        etpg, ekeys, eids = O.isect_tiles(as_np(meta["means2d"]), as_np(meta["radii"]),
                                          as_np(meta["depths"]), ts, tw, th, conics=as_np(meta["conics"]),
                                          opacities=as_np(meta["opacities"]))
    assert_equal(keys, ekeys, "isect_ids")
    assert_equal(meta["flatten_ids"], eids, "flatten_ids")
    assert_equal(meta["isect_offsets"].reshape(-1), O.isect_offset_encode(ekeys, 1, tw, th).reshape(-1),
                 "isect_offsets")
    if meta["tiles_per_gauss"] is not None:
        assert_equal(meta["tiles_per_gauss"].reshape(-1), np.asarray(etpg).reshape(-1), "tiles_per_gauss")
    # the buckets of this scene span the on-chip size classes
    sizes = np.bincount((ekeys >> 32).astype(np.int64))
    assert sizes.max() > 1024, sizes.max()
