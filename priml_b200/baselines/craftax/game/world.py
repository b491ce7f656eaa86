"""Overworld generation and the day / night cycle (``priml/baselines/craftax/game/world_gen.py``).

Terrain comes from fractal value noise: per world, random lattices at three
resolutions are upsampled bilinearly and summed (each octave half the weight of
the last), all batched over worlds. Four fields decide the tiles:

* ``water`` low -> lakes, a sand rim around them;
* ``mountain`` high -> stone, with caves (``cave`` field) carved as paths and
  lava pools in the highest parts, and ore scattered in the stone: coal (common),
  iron (near caves), diamond (rare, deep);
* ``forest`` high -> dense trees on grass, sparse trees elsewhere.

The player starts at the map centre on a cleared 3 x 3 patch of grass; a few
cows are placed on grass. The day length is 300 steps and
``daylight = 1 - |cos(pi * (t / 300 mod 1 + 0.3))|^3`` (Crafter's cycle: the
episode starts in the morning).
"""

from __future__ import annotations

import math

import torch
from torch import Tensor
from torch.nn import functional as F

from priml_b200.baselines.craftax.game import constants as C
from priml_b200.baselines.craftax.game.constants import BlockType as B
from priml_b200.baselines.craftax.game.state import GameState, empty_state

__all__ = ["daylight", "generate", "value_noise"]


def value_noise(envs: int, size: tuple[int, int], *, generator: torch.Generator | None, device: torch.device,
                octaves: tuple[int, ...] = (4, 8, 16)) -> Tensor:  # fmt: skip
    """``[envs, H, W]`` fractal value noise in about [-1, 1]: lattices of ``octaves`` cells per side."""
    out = torch.zeros(envs, 1, *size, device=device)
    weight, total = 1.0, 0.0
    for cells in octaves:
        lattice = torch.rand(envs, 1, cells + 1, cells + 1, device=device, generator=generator) * 2 - 1
        out += weight * F.interpolate(lattice, size=size, mode="bilinear", align_corners=True)
        total += weight
        weight *= 0.5
    return out[:, 0] / total


def daylight(t: Tensor) -> Tensor:
    progress = torch.remainder(t.float() / C.DAY_LENGTH, 1.0) + 0.3
    return 1.0 - torch.cos(math.pi * progress).abs() ** 3


def generate(envs: int, *, generator: torch.Generator | None, device: torch.device) -> GameState:
    rows, cols = C.MAP_SIZE
    s = empty_state(envs, device)

    def noise(octaves: tuple[int, ...] = (4, 8, 16)) -> Tensor:
        return value_noise(envs, (rows, cols), generator=generator, device=device, octaves=octaves)

    def uniform() -> Tensor:
        return torch.rand(envs, rows, cols, device=device, generator=generator)

    water, mountain, cave, forest = noise(), noise(), noise((6, 12)), noise((3, 6))
    ore = uniform()
    rr, cc = torch.meshgrid(torch.arange(rows, device=device), torch.arange(cols, device=device), indexing="ij")
    centre = ((rr - rows // 2).abs() + (cc - cols // 2).abs()).float()
    # keep the spawn region mostly land
    water = water + 0.5 * torch.clamp(1.0 - centre / 10.0, min=0.0)
    mountain = mountain - 0.5 * torch.clamp(1.0 - centre / 10.0, min=0.0)

    m = torch.full((envs, rows, cols), int(B.GRASS), dtype=torch.long, device=device)
    m = torch.where(water < -0.25, int(B.SAND), m)
    m = torch.where(water < -0.35, int(B.WATER), m)
    stone = (mountain > 0.18) & (water >= -0.25)
    m = torch.where(stone, int(B.STONE), m)
    m = torch.where(stone & (cave.abs() < 0.06), int(B.PATH), m)
    m = torch.where(stone & (mountain > 0.45) & (cave > 0.25), int(B.LAVA), m)
    near_cave = F.max_pool2d((m == int(B.PATH)).float()[:, None], 3, 1, 1)[:, 0] > 0
    rock = m == int(B.STONE)
    m = torch.where(rock & (ore < 0.07), int(B.COAL), m)
    m = torch.where(rock & near_cave & (ore > 0.96), int(B.IRON), m)
    m = torch.where(rock & (mountain > 0.35) & (ore > 0.994), int(B.DIAMOND), m)
    grass = m == int(B.GRASS)
    trees = uniform()
    m = torch.where(grass & (((forest > 0.15) & (trees < 0.35)) | (trees < 0.02)), int(B.TREE), m)

    # cleared spawn
    r0, c0 = rows // 2, cols // 2
    m[:, r0 - 1 : r0 + 2, c0 - 1 : c0 + 2] = int(B.GRASS)
    s.map = m
    s.position = torch.tensor([r0, c0], device=device).expand(envs, 2).clone()

    # a few cows on grass near the start
    for slot in range(C.MAX_PASSIVE_MOBS):
        pos = torch.stack([torch.randint(r0 - 8, r0 + 9, (envs,), device=device, generator=generator),
                           torch.randint(c0 - 8, c0 + 9, (envs,), device=device, generator=generator)], -1)  # fmt: skip
        on_grass = s.map.gather(1, pos[:, :1, None].expand(-1, 1, cols)).squeeze(1).gather(1, pos[:, 1:]).squeeze(1)
        ok = (on_grass == int(B.GRASS)) & ((pos - s.position).abs().sum(-1) > 1)
        s.passive.position[:, slot] = pos
        s.passive.mask[:, slot] = ok
        s.passive.health[:, slot] = C.PASSIVE_HEALTH
    s.light = daylight(s.timestep)
    return s
