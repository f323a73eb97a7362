"""Contribution bits of the raster forward and the backward that walks them
(tests/test_contribution_pruning.py:13-147, restated for the fp32
rasterizer's layout: one 32-bit word per (tile, batch of 32 pairs, 8-pixel-
wide warp block), word ((tile_start >> 5) + tile + batch) * warps + warp).

Each tile's Gaussians sit on the tile's first pixel centre (or cover the
whole tile when opaque), in tiles of 0, 31, 32, 33, 65 and 1 pairs on an
image whose right column and bottom row of tiles are clipped.  The words
the backward reads must hold exactly the contributing pairs; every word it
must not read (past a warp's last composited pair) is poisoned with ones and
the gradients stay bit-identical."""

import dataclasses

import numpy as np
import pytest

from tests.helpers import torch_proj

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

COUNTS = np.array([0, 31, 32, 33, 65, 1], np.int32)


def _case(kind, tile_h, tile_w, arena=256):
    from jaxgs_b200.scene import CapacityConfig
    from jaxgs_b200.types import DeviceCamera, SortedVisibilityTable

    offsets = np.concatenate([[0], np.cumsum(COUNTS)]).astype(np.int32)
    count = int(offsets[-1])
    width, height = tile_w + 3, tile_h * 2 + 1
    tile = np.repeat(np.arange(COUNTS.size), COUNTS)
    mean = np.stack((tile % 2 * tile_w, tile // 2 * tile_h), axis=1) + 0.5
    alpha = np.where(np.arange(count) % 2 == 0, 0.25, 0.001).astype(np.float32)
    if kind == "empty":
        alpha.fill(0)
    if kind == "opaque":
        alpha.fill(0.99)
    conic = np.eye(2, dtype=np.float32) * (0 if kind == "opaque" else 20)
    proj = {"mean": mean.astype(np.float32), "depth": np.arange(count, dtype=np.float32),
            "conic": np.broadcast_to(conic, (count, 2, 2)), "radius": np.ones(count, np.float32),
            "color": np.full((count, 3), 0.5, np.float32), "alpha": alpha,
            "visible": np.ones(count, np.int8)}
    ids = np.pad(np.arange(count, dtype=np.int32), (0, arena - count), constant_values=-1)
    table = SortedVisibilityTable(torch.as_tensor(ids, device="cuda"),
                                  torch.as_tensor(offsets, device="cuda"),
                                  torch.ones(count, dtype=torch.int32, device="cuda"),
                                  torch.tensor([count], dtype=torch.int32, device="cuda"),
                                  torch.tensor([0], dtype=torch.int32, device="cuda"))
    config = CapacityConfig(count, 128, 1, tile_w, 0, arena, tile_height=tile_h)
    camera = DeviceCamera(None, None, None, None, width, height)
    return torch_proj(proj), table, config, camera, offsets, alpha


def _expected(kind, offsets, alpha, tile_h, tile_w, width, height):
    """Per-pixel contributing pairs, restating the fp32 compositing rule
    (alpha >= 1/256, capped at 255/256; stop once T < 1/8192) for these
    splats: a 20 I conic reaches 1/256 only at the tile's first pixel."""
    contributes = {}
    for t in range(COUNTS.size):
        x0, y0 = t % 2 * tile_w, t // 2 * tile_h
        pixels = ([(x, y) for y in range(y0, min(y0 + tile_h, height))
                   for x in range(x0, min(x0 + tile_w, width))] if kind == "opaque"
                  else [(x0, y0)])
        for pixel in pixels:
            trans = np.float32(1)
            hits = []
            for i in range(offsets[t], offsets[t + 1]):
                a = np.float32(alpha[i])
                if a < np.float32(1 / 256):
                    continue
                a = min(a, np.float32(255 / 256))
                hits.append(i)
                trans = np.float32(trans * (np.float32(1) - a))
                if trans < np.float32(1 / 8192):
                    break
            contributes[pixel] = hits
    return contributes


def _warp_blocks(t, tile_h, tile_w, width, height):
    """(warp, [pixels in the image]) of tile t: 8 columns by 4 * rows each."""
    rows = 2 if tile_h % 8 == 0 else 1
    blocks_x = tile_w // 8
    warps = blocks_x * (tile_h // (4 * rows))
    x0, y0 = t % 2 * tile_w, t // 2 * tile_h
    out = []
    for w in range(warps):
        bx, by = x0 + w % blocks_x * 8, y0 + w // blocks_x * 4 * rows
        out.append((w, [(x, y) for y in range(by, min(by + 4 * rows, height))
                        for x in range(bx, min(bx + 8, width))]))
    return warps, out


def _same(a, b, exact):
    if exact:
        assert torch.equal(a, b)
    else:
        np.testing.assert_allclose(a.cpu().numpy(), b.cpu().numpy(), rtol=1e-6, atol=0)


@pytest.mark.parametrize("kind", ["holes", "empty", "opaque"])
@pytest.mark.parametrize("collect_stats", [False, True])
@pytest.mark.parametrize("tile_h,tile_w", [(8, 8), (8, 16), (12, 16), (16, 16)])
def test_contribution_bits_and_backward_ignore_unread_words(kind, collect_stats, tile_h, tile_w):
    from jaxgs_b200 import kernels as K

    projected, table, config, camera, offsets, alpha = _case(kind, tile_h, tile_w)
    width, height = camera.width, camera.height
    result, cache = K.rasterize_forward(projected, table, camera, config)
    image_only, none = K.rasterize_forward(projected, table, camera, config, record=False)
    torch.cuda.synchronize()
    assert none is None
    assert torch.equal(image_only.rgb, result.rgb)

    contributes = _expected(kind, offsets, alpha, tile_h, tile_w, width, height)
    count = int(offsets[-1])
    expected = np.zeros(count, bool)
    for hits in contributes.values():
        expected[hits] = True
    if kind != "empty":
        assert expected.any() and not expected.all()

    bits = cache.contribution_bits.cpu().numpy().view(np.uint32)
    last = cache.last.cpu().numpy().reshape(height, width)
    poisoned = np.full_like(bits, 0xFFFFFFFF)
    read_words = 0
    for t in range(COUNTS.size):
        start, end = int(offsets[t]), int(offsets[t + 1])
        warps, blocks = _warp_blocks(t, tile_h, tile_w, width, height)
        for w, pixels in blocks:
            top = max([int(last[y, x]) for x, y in pixels], default=start)
            if top <= start:
                continue
            top_batch = (top - 1 - start) >> 5
            for batch in range(top_batch + 1):
                word = ((start >> 5) + t + batch) * warps + w
                want = 0
                for x, y in pixels:
                    for i in contributes.get((x, y), []):
                        if start + batch * 32 <= i < min(start + batch * 32 + 32, top):
                            want |= 1 << (i - start - batch * 32)
                got = int(bits[word])
                keep = 0xFFFFFFFF
                if batch == top_batch:
                    keep = (2 << ((top - 1 - start) & 31)) - 1 & 0xFFFFFFFF
                assert got & keep == want, (t, w, batch, hex(got), hex(want))
                poisoned[word] = (got & keep) | (~keep & 0xFFFFFFFF)
                read_words += 1
    assert read_words > 0

    # One warp composites each Gaussian unless opaque, so only then do
    # several warps' float atomics meet (in either order).
    exact = kind != "opaque"
    incoming = torch.tensor([1.0, -1.0, 0.0], device="cuda").expand(height, width, 3).contiguous()
    grads = K.rasterize_backward(projected, table, cache, incoming, camera, config,
                                 collect_stats=collect_stats)
    poisoned_cache = dataclasses.replace(
        cache, contribution_bits=torch.as_tensor(poisoned.view(np.int32), device="cuda"))
    other = K.rasterize_backward(projected, table, poisoned_cache, incoming, camera, config,
                                 collect_stats=collect_stats)
    torch.cuda.synchronize()
    if collect_stats:
        grads, stats = grads
        other, other_stats = other
        pixel_counts = np.zeros(count, np.float32)
        for hits in contributes.values():
            pixel_counts[hits] += 1
        np.testing.assert_array_equal(stats[:, 0].cpu().numpy(), pixel_counts)
        _same(stats, other_stats, exact)
    for field in ("mean", "conic", "color", "alpha"):
        _same(getattr(grads, field), getattr(other, field), exact)
    # Equal R/G colours cancel the opacity and geometry cotangents exactly,
    # not the colour ones.
    for field in ("mean", "conic", "alpha"):
        assert float(getattr(grads, field).abs().max()) == 0, field
    color = grads.color.cpu().numpy()
    np.testing.assert_array_equal(color[:, 0] > 0, expected)
    np.testing.assert_allclose(color[:, 1], -color[:, 0], rtol=0 if exact else 1e-6, atol=0)
    np.testing.assert_array_equal(color[:, 2], 0)


@pytest.mark.parametrize("tile_h,tile_w", [(8, 8), (8, 16), (12, 16), (16, 16)])
def test_empty_pixel_groups_preserve_accumulated_gradients(tile_h, tile_w):
    """tests/test_contribution_pruning.py:150-188: narrow splats that each hit
    one pixel group leave the tile's other groups empty before and after a
    nonzero partial gradient; the backward with fragment statistics gives
    the same cotangents as the plain one."""
    from jaxgs_b200 import kernels as K
    from jaxgs_b200.scene import CapacityConfig
    from jaxgs_b200.types import DeviceCamera, SortedVisibilityTable

    count = 65
    width, height = tile_w + 3, tile_h + 1
    rows = 2 if tile_h % 8 == 0 else 1
    groups = (tile_w // 8) * (tile_h // (4 * rows))
    rng = np.random.default_rng(14)
    mean = np.stack((np.arange(count) % 3 * 2 + 0.7,
                     np.arange(count) % groups * 4 * rows % tile_h + 0.4), 1)
    proj = {"mean": mean.astype(np.float32), "depth": np.arange(count, dtype=np.float32),
            "conic": np.broadcast_to(np.eye(2, dtype=np.float32) * 20, (count, 2, 2)),
            "radius": np.ones(count, np.float32),
            "color": rng.random((count, 3)).astype(np.float32),
            "alpha": np.where(np.arange(count) % 5 == 0, 0.001, 0.3).astype(np.float32),
            "visible": np.ones(count, np.int8)}
    tiles = 2 * 2
    offsets = np.array([0] + [count] * tiles, np.int32)
    ids = np.pad(np.arange(count, dtype=np.int32), (0, 96 - count), constant_values=-1)
    table = SortedVisibilityTable(torch.as_tensor(ids, device="cuda"),
                                  torch.as_tensor(offsets, device="cuda"),
                                  torch.ones(count, dtype=torch.int32, device="cuda"),
                                  torch.tensor([count], dtype=torch.int32, device="cuda"),
                                  torch.tensor([0], dtype=torch.int32, device="cuda"))
    config = CapacityConfig(count, 128, 1, tile_w, 0, 96, tile_height=tile_h)
    camera = DeviceCamera(None, None, None, None, width, height)
    projected = torch_proj(proj)
    result, cache = K.rasterize_forward(projected, table, camera, config)
    incoming = torch.as_tensor(rng.normal(size=(height, width, 3)).astype(np.float32),
                               device="cuda")
    ordinary = K.rasterize_backward(projected, table, cache, incoming, camera, config)
    with_stats, _ = K.rasterize_backward(projected, table, cache, incoming, camera, config,
                                         collect_stats=True)
    torch.cuda.synchronize()
    for field in ("mean", "conic", "color", "alpha"):
        expected = getattr(with_stats, field).cpu().numpy()
        assert np.any(expected != 0), field
        np.testing.assert_allclose(getattr(ordinary, field).cpu().numpy(), expected,
                                   rtol=1e-5, atol=1e-8)
