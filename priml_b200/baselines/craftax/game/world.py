"""World generation for all nine floors and the day / night cycle (``priml/baselines/craftax/game/world_gen.py``).

Terrain comes from fractal value noise: per world, random lattices at three
resolutions are upsampled bilinearly and summed (each octave half the weight of
the last), all batched over worlds. Four fields decide the tiles:

* ``water`` low -> lakes, a sand rim around them;
* ``mountain`` high -> stone, with caves (``cave`` field) carved as paths and
  lava pools in the highest parts, and ore scattered in the stone: coal (common),
  iron (near caves), diamond (rare, deep);
* ``forest`` high -> dense trees on grass, sparse trees elsewhere.

The player starts at the map centre on a cleared 3 x 3 patch of grass; a few
cows are placed on grass and a ladder down lies on grass 6-12 steps away. The
floors below are this build's own layouts: the dungeon, sewers (water channels)
and vault (a chest in every room, both enchantment tables) are walls with eight
rectangular rooms joined by L-shaped corridors, a fountain and the ladders in
the first and last rooms; the gnomish and troll mines (the latter with lava)
are stone with noise-carved tunnels and ores including sapphire and ruby; the
fire and ice realms are open ground with lava / water pools, fire trees / ice
shrubs and the realm's enchantment table; the graveyard is grass with graves,
the necromancer and no ladder down. Ladders on cave and open floors are joined
by a cleared path. The day length is 300 steps and
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
from priml_b200.baselines.craftax.game.constants import ItemType as I
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

    # ladder down to the dungeon on a grass tile 6..12 steps from the start
    for _ in range(8):
        cand = torch.stack([r0 + torch.randint(-12, 13, (envs,), device=device, generator=generator),
                            c0 + torch.randint(-12, 13, (envs,), device=device, generator=generator)], -1)  # fmt: skip
        d = (cand - s.position).abs().sum(-1)
        ok = (_at(m, cand) == int(B.GRASS)) & (d >= 6)
        unset = (s.ladder_down[:, 0] == 0).all(-1)
        s.ladder_down[:, 0] = torch.where((ok & unset)[:, None], cand, s.ladder_down[:, 0])
    unset = (s.ladder_down[:, 0] == 0).all(-1)
    s.ladder_down[:, 0] = torch.where(unset[:, None], s.position + torch.tensor([0, 2], device=device), s.ladder_down[:, 0])
    e = torch.arange(envs, device=device)
    m[e, s.ladder_down[:, 0, 0], s.ladder_down[:, 0, 1]] = int(B.GRASS)
    s.item_map[e, s.ladder_down[:, 0, 0], s.ladder_down[:, 0, 1]] = int(I.LADDER_DOWN)
    s.map = m

    s.floor_map[:, 0], s.floor_items[:, 0] = m, s.item_map
    for level in range(1, C.LEVELS):
        fm, fi, up, down = _FLOORS[level](envs, generator=generator, device=device)
        if level == C.LEVELS - 1:  # the deepest floor has no way down
            fi = torch.where(fi == int(I.LADDER_DOWN), int(I.NONE), fi)
        s.floor_map[:, level], s.floor_items[:, level] = fm, fi
        s.ladder_up[:, level], s.ladder_down[:, level] = up, down
    _furnish(s)
    s.visited[:, 0] = True
    s.potion_effect = torch.rand(envs, 6, device=device, generator=generator).argsort(-1)

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


def _at(grid: Tensor, pos: Tensor) -> Tensor:
    rows, cols = grid.shape[-2:]
    p0, p1 = pos[:, 0].clamp(0, rows - 1), pos[:, 1].clamp(0, cols - 1)
    return grid[torch.arange(grid.shape[0], device=grid.device), p0, p1]


def _dungeon(envs: int, *, generator: torch.Generator | None, device: torch.device, rooms: int = 8,
             chest_prob: float = 0.5, water: bool = False) -> tuple[Tensor, Tensor, Tensor, Tensor]:  # fmt: skip
    """Walled floor with ``rooms`` rectangular rooms joined in sequence by L-shaped corridors;
    chests in rooms with probability ``chest_prob``, a fountain in one, water channels down the
    corridors' side when ``water``, the ladder up in the first room's centre and the ladder down
    in the last one's."""
    rows, cols = C.MAP_SIZE

    def ri(lo: int, hi: int) -> Tensor:
        return torch.randint(lo, hi, (envs, rooms), device=device, generator=generator)

    h, w = ri(4, 9), ri(4, 9)
    top, left = ri(1, rows - 10), ri(1, cols - 10)
    rr = torch.arange(rows, device=device).view(1, 1, rows, 1)
    cc = torch.arange(cols, device=device).view(1, 1, 1, cols)
    inside = (rr >= top[..., None, None]) & (rr < (top + h)[..., None, None]) & \
             (cc >= left[..., None, None]) & (cc < (left + w)[..., None, None])  # fmt: skip
    open_ = inside.any(1)
    cr, cc_ = top + h // 2, left + w // 2  # room centres
    for k in range(rooms - 1):
        a_r, a_c, b_r, b_c = cr[:, k], cc_[:, k], cr[:, k + 1], cc_[:, k + 1]
        row = rr[0, 0, :, 0]
        col = cc[0, 0, 0, :]
        horiz = (row[None, :, None] == a_r[:, None, None]) & \
                (col[None, None, :] >= torch.minimum(a_c, b_c)[:, None, None]) & \
                (col[None, None, :] <= torch.maximum(a_c, b_c)[:, None, None])  # fmt: skip
        vert = (col[None, None, :] == b_c[:, None, None]) & \
               (row[None, :, None] >= torch.minimum(a_r, b_r)[:, None, None]) & \
               (row[None, :, None] <= torch.maximum(a_r, b_r)[:, None, None])  # fmt: skip
        open_ |= horiz | vert
    m = torch.where(open_, int(B.PATH), int(B.WALL))
    if water:  # sewer channels: open tiles beside walls on even rows flood
        beside = F.max_pool2d((m == int(B.WALL)).float()[:, None], 3, 1, 1)[:, 0] > 0
        m = torch.where(open_ & ~inside.any(1) & beside & (rr[0, 0] % 2 == 0), int(B.WATER), m)
    e = torch.arange(envs, device=device)
    # chests in rooms 1..rooms-2, at the room's top-left interior tile
    for k in range(1, rooms - 1):
        put = torch.rand(envs, device=device, generator=generator) < chest_prob
        pr, pc = top[:, k], left[:, k]
        m[e, pr, pc] = torch.where(put, int(B.CHEST), m[e, pr, pc])
    m[e, top[:, 1] + h[:, 1] - 1, left[:, 1] + w[:, 1] - 1] = int(B.FOUNTAIN)
    items = torch.zeros_like(m)
    up = torch.stack([cr[:, 0], cc_[:, 0]], -1)
    down = torch.stack([cr[:, -1], cc_[:, -1]], -1)
    m[e, up[:, 0], up[:, 1]] = int(B.PATH)
    m[e, down[:, 0], down[:, 1]] = int(B.PATH)
    items[e, up[:, 0], up[:, 1]] = int(I.LADDER_UP)
    items[e, down[:, 0], down[:, 1]] = int(I.LADDER_DOWN)
    return m, items, up, down


def _ladders(envs: int, m: Tensor, *, generator: torch.Generator | None,
             device: torch.device) -> tuple[Tensor, Tensor, Tensor, Tensor]:  # fmt: skip
    """Ladders far apart, joined by a cleared L-shaped path so that the floor can be crossed."""
    rows, cols = C.MAP_SIZE
    up = torch.stack([torch.randint(4, rows - 4, (envs,), device=device, generator=generator),
                      torch.randint(4, cols // 3, (envs,), device=device, generator=generator)], -1)  # fmt: skip
    down = torch.stack([torch.randint(4, rows - 4, (envs,), device=device, generator=generator),
                        torch.randint(2 * cols // 3, cols - 4, (envs,), device=device, generator=generator)], -1)  # fmt: skip
    rr = torch.arange(rows, device=device).view(1, rows, 1)
    cc = torch.arange(cols, device=device).view(1, 1, cols)
    lo_c, hi_c = torch.minimum(up[:, 1], down[:, 1]), torch.maximum(up[:, 1], down[:, 1])
    lo_r, hi_r = torch.minimum(up[:, 0], down[:, 0]), torch.maximum(up[:, 0], down[:, 0])
    path = ((rr == up[:, 0, None, None]) & (cc >= lo_c[:, None, None]) & (cc <= hi_c[:, None, None])) | \
           ((cc == down[:, 1, None, None]) & (rr >= lo_r[:, None, None]) & (rr <= hi_r[:, None, None]))  # fmt: skip
    e = torch.arange(envs, device=device)
    items = torch.zeros_like(m)
    items[e, up[:, 0], up[:, 1]] = int(I.LADDER_UP)
    items[e, down[:, 0], down[:, 1]] = int(I.LADDER_DOWN)
    return m, path, up, down, items  # type: ignore[return-value]


def _cave(envs: int, *, generator: torch.Generator | None, device: torch.device, lava: bool,
          ores: tuple[float, float, float, float, float]) -> tuple[Tensor, Tensor, Tensor, Tensor]:  # fmt: skip
    """Stone with noise-carved tunnels; ore probabilities (coal, iron, diamond, sapphire, ruby)."""
    rows, cols = C.MAP_SIZE
    n = value_noise(envs, (rows, cols), generator=generator, device=device, octaves=(6, 12))
    m = torch.where(n.abs() < 0.18, int(B.PATH), int(B.STONE))
    u = torch.rand(envs, rows, cols, device=device, generator=generator)
    rock = m == int(B.STONE)
    edge = 0.0
    for block, p in zip((B.COAL, B.IRON, B.DIAMOND, B.SAPPHIRE, B.RUBY), ores, strict=True):
        m = torch.where(rock & (u >= edge) & (u < edge + p), int(block), m)
        edge += p
    if lava:
        m = torch.where((m == int(B.PATH)) & (n > 0.12) & (u > 0.9), int(B.LAVA), m)
    m, path, up, down, items = _ladders(envs, m, generator=generator, device=device)
    m = torch.where(path, int(B.PATH), m)
    return m, items, up, down


def _realm(envs: int, *, generator: torch.Generator | None, device: torch.device, ground: B, hazard: B,
           flora: B, extra: B | None = None) -> tuple[Tensor, Tensor, Tensor, Tensor]:  # fmt: skip
    """Open floor of ``ground`` with ``hazard`` pools, ``flora`` scattered, ``extra`` blocks sparse."""
    rows, cols = C.MAP_SIZE
    n = value_noise(envs, (rows, cols), generator=generator, device=device)
    u = torch.rand(envs, rows, cols, device=device, generator=generator)
    m = torch.full((envs, rows, cols), int(ground), dtype=torch.long, device=device)
    m = torch.where(n < -0.3, int(hazard), m)
    m = torch.where((m == int(ground)) & (u < 0.08), int(flora), m)
    if extra is not None:
        m = torch.where((m == int(ground)) & (u > 0.985), int(extra), m)
    m, path, up, down, items = _ladders(envs, m, generator=generator, device=device)
    m = torch.where(path, int(ground), m)
    return m, items, up, down


def _graveyard(envs: int, *, generator: torch.Generator | None,
               device: torch.device) -> tuple[Tensor, Tensor, Tensor, Tensor]:  # fmt: skip
    rows, cols = C.MAP_SIZE
    u = torch.rand(envs, rows, cols, device=device, generator=generator)
    m = torch.full((envs, rows, cols), int(B.GRASS), dtype=torch.long, device=device)
    for block, lo in ((B.GRAVE, 0.0), (B.GRAVE2, 0.02), (B.GRAVE3, 0.04)):
        m = torch.where((u >= lo) & (u < lo + 0.02), int(block), m)
    m, path, up, down, items = _ladders(envs, m, generator=generator, device=device)
    m = torch.where(path, int(B.GRASS), m)
    return m, items, up, down


def _furnish(s: GameState) -> None:
    """Enchantment tables beside the ladder up (both in the vault, the fire one in the fire realm,
    the ice one in the ice realm) and the necromancer in the graveyard's centre column."""
    e = torch.arange(s.num_envs, device=s.device)
    for level, tables in ((4, (B.ENCHANTMENT_TABLE_FIRE, B.ENCHANTMENT_TABLE_ICE)), (6, (B.ENCHANTMENT_TABLE_FIRE,)),
                          (7, (B.ENCHANTMENT_TABLE_ICE,))):  # fmt: skip
        up = s.ladder_up[:, level]
        for side, table in zip((-1, 1), tables, strict=False):
            s.floor_map[e, level, up[:, 0] - 1, up[:, 1] + side] = int(table)
    last = C.LEVELS - 1
    rows, cols = C.MAP_SIZE
    boss_r = torch.where(s.ladder_up[:, last, 0] == rows // 2, rows // 2 - 4, rows // 2)
    for dr in (-1, 0, 1):
        for dc in (-1, 0, 1):
            s.floor_map[e, last, boss_r + dr, cols // 2 + dc] = int(B.GRASS)
    s.floor_map[e, last, boss_r, cols // 2] = int(B.NECROMANCER)


_FLOORS = {
    1: _dungeon,
    2: lambda envs, **kw: _cave(envs, lava=False, ores=(0.06, 0.04, 0.01, 0.008, 0.008), **kw),
    3: lambda envs, **kw: _dungeon(envs, water=True, **kw),
    4: lambda envs, **kw: _dungeon(envs, chest_prob=1.0, **kw),
    5: lambda envs, **kw: _cave(envs, lava=True, ores=(0.04, 0.04, 0.015, 0.01, 0.01), **kw),
    6: lambda envs, **kw: _realm(envs, ground=B.FIRE_GRASS, hazard=B.LAVA, flora=B.FIRE_TREE, extra=B.RUBY, **kw),
    7: lambda envs, **kw: _realm(envs, ground=B.ICE_GRASS, hazard=B.WATER, flora=B.ICE_SHRUB, extra=B.SAPPHIRE, **kw),
    8: _graveyard,
}
"""Floor generators below the surface (this build's layouts)."""
