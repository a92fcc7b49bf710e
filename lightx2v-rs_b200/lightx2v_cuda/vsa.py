"""Video sparse attention geometry, restating crates/lightx2v-core/src/sparse.rs
(the plan the reference's sparse_prepare receives): the (T, H, W) token grid
tiled into 4 x 4 x 4 cubes of 64 slots, a partial cube filling its first
slots; topk_for; SparseSpec's topk and scale. The C ABI's lx2v_sparse_prepare
takes this plan as is, so a Rust caller passes its own TilePlan unchanged."""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

TILE = (4, 4, 4)
TILE_ELEMS = 64
PAD = 0xFFFFFFFF
DEFAULT_SPARSITY = 0.8


def topk_for(sparsity: float, num_tiles: int) -> int:
    """sparse.rs:27-30: ceil((1 - sparsity) * tiles), clamped to [1, tiles]."""
    return min(max(int(math.ceil((1.0 - sparsity) * num_tiles)), 1), max(num_tiles, 1))


@dataclass
class TilePlan:
    grid: tuple
    tiles: tuple
    seq: int
    slot_src: np.ndarray      # u32 [num_tiles * 64]
    block_sizes: np.ndarray   # u32 [num_tiles]

    @staticmethod
    def new(grid) -> "TilePlan":
        """sparse.rs:45-78: tiles in (t, h, w) order, slots in (z, y, x) order."""
        t, h, w = grid
        ts, hs, ws = TILE
        tiles = (-(-t // ts), -(-h // hs), -(-w // ws))
        nb = tiles[0] * tiles[1] * tiles[2]
        slot_src = np.full(nb * TILE_ELEMS, PAD, np.uint32)
        sizes = np.zeros(nb, np.uint32)
        tile = 0
        for tt in range(tiles[0]):
            for hh in range(tiles[1]):
                for ww in range(tiles[2]):
                    slot = tile * TILE_ELEMS
                    for z in range(tt * ts, min((tt + 1) * ts, t)):
                        for y in range(hh * hs, min((hh + 1) * hs, h)):
                            for x in range(ww * ws, min((ww + 1) * ws, w)):
                                slot_src[slot] = (z * h + y) * w + x
                                slot += 1
                    sizes[tile] = slot - tile * TILE_ELEMS
                    tile += 1
        return TilePlan(tuple(grid), tiles, t * h * w, slot_src, sizes)

    def num_tiles(self) -> int:
        return int(self.block_sizes.size)


@dataclass
class SparseSpec:
    plan: TilePlan
    heads: int
    head_dim: int
    topk: int
    scale: float

    @staticmethod
    def new(grid, heads: int, head_dim: int, sparsity: float) -> "SparseSpec":
        plan = TilePlan.new(grid)
        return SparseSpec(plan, heads, head_dim, topk_for(sparsity, plan.num_tiles()),
                          float(np.float32(1.0) / np.sqrt(np.float32(head_dim))))
