"""Symbolic observation of the Craftax game (``priml/baselines/craftax/game/observation.py``).

Per visible tile of the 9 x 11 local view: a one-hot block (37 planes), a
one-hot item (5), creature planes (5 classes x 8 species: passive, melee,
ranged, mob projectile, player projectile) and a lit flag -- 83 planes, masked
by the lit flag -- flattened, then 51 player features (square-rooted counts,
tool levels, meters / 10, facing direction, armour, condition). 8,268 floats
in all, the same layout as the reference so that trained networks read it.
Tiles beyond the map edge read OUT_OF_BOUNDS. The overworld is always lit; in
the dungeon a tile is seen within 3 tiles of the player or 4 of a torch (this
build's light rule).
"""

from __future__ import annotations

import torch
from torch import Tensor
from torch.nn import functional as F

from priml_b200.baselines.craftax.game import constants as C
from priml_b200.baselines.craftax.game.state import GameState

__all__ = ["CHANNELS_PER_TILE", "local_view", "observation_size", "render", "visible_tiles"]

CHANNELS_PER_TILE = len(C.BlockType) + len(C.ItemType) + 5 * 8 + 1


def observation_size(view: tuple[int, int] = C.OBS_DIM) -> int:
    return view[0] * view[1] * CHANNELS_PER_TILE + C.INVENTORY_OBS_SIZE


def _local(grid: Tensor, pos: Tensor, view: tuple[int, int], outside: int) -> Tensor:
    vr, vc = view
    pad = max(vr, vc)
    padded = F.pad(grid, (pad, pad, pad, pad), value=outside)
    r0 = pos[:, 0] - vr // 2 + pad
    c0 = pos[:, 1] - vc // 2 + pad
    rr = r0[:, None] + torch.arange(vr, device=grid.device)
    cc = c0[:, None] + torch.arange(vc, device=grid.device)
    e = torch.arange(grid.shape[0], device=grid.device)
    return padded[e[:, None, None], rr[:, :, None], cc[:, None, :]]


def local_view(s: GameState, view: tuple[int, int] = C.OBS_DIM) -> tuple[Tensor, Tensor]:
    """``(blocks, items)`` of the ``view`` window centred on the player (``[E, rows, cols]``)."""
    blocks = _local(s.map, s.position, view, int(C.BlockType.OUT_OF_BOUNDS))
    items = _local(s.item_map, s.position, view, int(C.ItemType.NONE))
    return blocks, items


def visible_tiles(s: GameState, items: Tensor, view: tuple[int, int] = C.OBS_DIM) -> Tensor:
    """``[E, rows, cols]`` bool: lit floors are seen whole; elsewhere 3 tiles around the player, 4 around a torch."""
    vr, vc = view
    rr = torch.arange(vr, device=s.device)[:, None] - vr // 2
    cc = torch.arange(vc, device=s.device)[None, :] - vc // 2
    near = (torch.maximum(rr.abs(), cc.abs()) <= 3).expand(s.num_envs, vr, vc)
    torch_light = F.max_pool2d((items == int(C.ItemType.TORCH)).float()[:, None], 9, 1, 4)[:, 0] > 0
    lit_floor = C.device_table("lit", s.device, C.LIT_FLOORS)[s.level]
    return lit_floor[:, None, None] | near | torch_light


def render(s: GameState, view: tuple[int, int] = C.OBS_DIM) -> Tensor:
    vr, vc = view
    blocks, items = local_view(s, view)
    mobs = torch.zeros(s.num_envs, vr, vc, 5 * 8, device=s.device)
    corner = s.position - C.device_table(("half", vr, vc), s.device, [vr // 2, vc // 2])
    e = torch.arange(s.num_envs, device=s.device)
    species = C.device_table("species", s.device, C.FLOOR_SPECIES)[s.level]  # [E, 3] per class
    for creatures, plane, cls in ((s.melee, 1, 1), (s.passive, 0, 0), (s.ranged, 2, 2),
                                  (s.projectiles, 3, 2), (s.shots, 4, None)):  # fmt: skip
        channel = plane * 8 + (species[:, cls] if cls is not None else torch.zeros_like(s.level))
        for slot in range(creatures.mask.shape[1]):
            local = creatures.position[:, slot] - corner
            seen = creatures.mask[:, slot] & (local[:, 0] >= 0) & (local[:, 0] < vr) & (local[:, 1] >= 0) & (local[:, 1] < vc)
            r, c = local[:, 0].clamp(0, vr - 1), local[:, 1].clamp(0, vc - 1)
            mobs[e, r, c, channel] = torch.maximum(mobs[e, r, c, channel], seen.float())
    lit = visible_tiles(s, items, view).float()[..., None]
    tiles = torch.cat([F.one_hot(blocks, len(C.BlockType)).float(), F.one_hot(items, len(C.ItemType)).float(), mobs], -1)
    view_part = torch.cat([tiles * lit, lit], -1).flatten(1)
    z = torch.zeros(s.num_envs, device=s.device)
    counts = torch.stack([s.wood, s.stone, s.coal, s.iron, s.diamond, s.sapphire, s.ruby, s.sapling, s.torches, s.arrows], -1).float()
    tools = torch.stack([s.books.float() / 2.0, s.pickaxe.float() / 4.0, s.sword.float() / 4.0, s.sword_enchant.float(),
                         s.bow_enchant.float(), s.bow.float()], -1)  # fmt: skip
    potions = s.potions.float().sqrt() / 10.0
    meters = torch.stack([s.health, s.food.float(), s.drink.float(), s.energy.float(), s.mana.float(), s.xp.float(),
                          s.dexterity.float(), s.strength.float(), s.intelligence.float()], -1)  # fmt: skip
    facing = F.one_hot((s.direction - 1).clamp(min=0), 4).float()
    cleared = (s.kills[e, s.level] >= C.MONSTERS_KILLED_TO_CLEAR_LEVEL).float()
    last = s.level == C.LEVELS - 1
    vulnerable = last & ~s.melee.mask.any(-1) & ~s.ranged.mask.any(-1) & (s.boss_wait <= 0)
    condition = torch.stack([s.light, s.sleeping.float(), s.resting.float(), s.spells[:, 0].float(), s.spells[:, 1].float(),
                             s.level.float() / 10.0, cleared, vulnerable.float()], -1)  # fmt: skip
    player = torch.cat([counts.sqrt() / 10.0, tools, potions, meters / 10.0, facing, s.armour.float() / 2.0,
                        s.armour_enchant.float(), condition], -1)  # fmt: skip
    return torch.cat([view_part, player], -1)
