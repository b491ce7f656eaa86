"""Vocabularies and tables of the Craftax game (``priml/baselines/craftax/game/constants.py``).

The enumerations (block, item, action, mob class, achievement) and their integer
values define the action space and the symbolic observation, so they are the
game's own and kept identical; the achievement rewards (1, 3, 5 or 8 by tier,
summing to 226) define the score. Craftax is Matthews et al. 2024
(arXiv:2402.16801, MIT licence), built on Crafter (Hafner 2021).
"""

from __future__ import annotations

from enum import IntEnum
from typing import Final

import torch


class BlockType(IntEnum):
    INVALID = 0
    OUT_OF_BOUNDS = 1
    GRASS = 2
    WATER = 3
    STONE = 4
    TREE = 5
    WOOD = 6
    PATH = 7
    COAL = 8
    IRON = 9
    DIAMOND = 10
    CRAFTING_TABLE = 11
    FURNACE = 12
    SAND = 13
    LAVA = 14
    PLANT = 15
    RIPE_PLANT = 16
    WALL = 17
    DARKNESS = 18
    WALL_MOSS = 19
    STALAGMITE = 20
    SAPPHIRE = 21
    RUBY = 22
    CHEST = 23
    FOUNTAIN = 24
    FIRE_GRASS = 25
    ICE_GRASS = 26
    GRAVEL = 27
    FIRE_TREE = 28
    ICE_SHRUB = 29
    ENCHANTMENT_TABLE_FIRE = 30
    ENCHANTMENT_TABLE_ICE = 31
    NECROMANCER = 32
    GRAVE = 33
    GRAVE2 = 34
    GRAVE3 = 35
    NECROMANCER_VULNERABLE = 36


class ItemType(IntEnum):
    NONE = 0
    TORCH = 1
    LADDER_DOWN = 2
    LADDER_UP = 3
    LADDER_DOWN_BLOCKED = 4


class Action(IntEnum):
    NOOP = 0
    LEFT = 1
    RIGHT = 2
    UP = 3
    DOWN = 4
    DO = 5
    SLEEP = 6
    PLACE_STONE = 7
    PLACE_TABLE = 8
    PLACE_FURNACE = 9
    PLACE_PLANT = 10
    MAKE_WOOD_PICKAXE = 11
    MAKE_STONE_PICKAXE = 12
    MAKE_IRON_PICKAXE = 13
    MAKE_WOOD_SWORD = 14
    MAKE_STONE_SWORD = 15
    MAKE_IRON_SWORD = 16
    REST = 17
    DESCEND = 18
    ASCEND = 19
    MAKE_DIAMOND_PICKAXE = 20
    MAKE_DIAMOND_SWORD = 21
    MAKE_IRON_ARMOUR = 22
    MAKE_DIAMOND_ARMOUR = 23
    SHOOT_ARROW = 24
    MAKE_ARROW = 25
    CAST_FIREBALL = 26
    CAST_ICEBALL = 27
    PLACE_TORCH = 28
    DRINK_POTION_RED = 29
    DRINK_POTION_GREEN = 30
    DRINK_POTION_BLUE = 31
    DRINK_POTION_PINK = 32
    DRINK_POTION_CYAN = 33
    DRINK_POTION_YELLOW = 34
    READ_BOOK = 35
    ENCHANT_SWORD = 36
    ENCHANT_ARMOUR = 37
    MAKE_TORCH = 38
    LEVEL_UP_DEXTERITY = 39
    LEVEL_UP_STRENGTH = 40
    LEVEL_UP_INTELLIGENCE = 41
    ENCHANT_BOW = 42


class MobClass(IntEnum):
    PASSIVE = 0
    MELEE = 1
    RANGED = 2
    MOB_PROJECTILE = 3
    PLAYER_PROJECTILE = 4


class Achievement(IntEnum):
    COLLECT_WOOD = 0
    PLACE_TABLE = 1
    EAT_COW = 2
    COLLECT_SAPLING = 3
    COLLECT_DRINK = 4
    MAKE_WOOD_PICKAXE = 5
    MAKE_WOOD_SWORD = 6
    PLACE_PLANT = 7
    DEFEAT_ZOMBIE = 8
    COLLECT_STONE = 9
    PLACE_STONE = 10
    EAT_PLANT = 11
    DEFEAT_SKELETON = 12
    MAKE_STONE_PICKAXE = 13
    MAKE_STONE_SWORD = 14
    WAKE_UP = 15
    PLACE_FURNACE = 16
    COLLECT_COAL = 17
    COLLECT_IRON = 18
    COLLECT_DIAMOND = 19
    MAKE_IRON_PICKAXE = 20
    MAKE_IRON_SWORD = 21
    MAKE_ARROW = 22
    MAKE_TORCH = 23
    PLACE_TORCH = 24
    MAKE_DIAMOND_SWORD = 25
    MAKE_IRON_ARMOUR = 26
    MAKE_DIAMOND_ARMOUR = 27
    ENTER_GNOMISH_MINES = 28
    ENTER_DUNGEON = 29
    ENTER_SEWERS = 30
    ENTER_VAULT = 31
    ENTER_TROLL_MINES = 32
    ENTER_FIRE_REALM = 33
    ENTER_ICE_REALM = 34
    ENTER_GRAVEYARD = 35
    DEFEAT_GNOME_WARRIOR = 36
    DEFEAT_GNOME_ARCHER = 37
    DEFEAT_ORC_SOLIDER = 38
    DEFEAT_ORC_MAGE = 39
    DEFEAT_LIZARD = 40
    DEFEAT_KOBOLD = 41
    DEFEAT_TROLL = 42
    DEFEAT_DEEP_THING = 43
    DEFEAT_PIGMAN = 44
    DEFEAT_FIRE_ELEMENTAL = 45
    DEFEAT_FROST_TROLL = 46
    DEFEAT_ICE_ELEMENTAL = 47
    DAMAGE_NECROMANCER = 48
    DEFEAT_NECROMANCER = 49
    EAT_BAT = 50
    EAT_SNAIL = 51
    FIND_BOW = 52
    FIRE_BOW = 53
    COLLECT_SAPPHIRE = 54
    LEARN_FIREBALL = 55
    CAST_FIREBALL = 56
    LEARN_ICEBALL = 57
    CAST_ICEBALL = 58
    COLLECT_RUBY = 59
    MAKE_DIAMOND_PICKAXE = 60
    OPEN_CHEST = 61
    DRINK_POTION = 62
    ENCHANT_SWORD = 63
    ENCHANT_ARMOUR = 64
    DEFEAT_KNIGHT = 65
    DEFEAT_ARCHER = 66


NUM_ACHIEVEMENTS: Final = len(Achievement)
OBS_DIM: Final = (9, 11)
"""Rows and columns of the local view."""
INVENTORY_OBS_SIZE: Final = 51
"""Scalar features appended to the flattened view."""
MAP_SIZE: Final = (48, 48)
DAY_LENGTH: Final = 300
MAX_TIMESTEPS: Final = 100_000
MAX_METER: Final = 9
"""Health, food, drink and energy saturate here."""
MAX_PASSIVE_MOBS: Final = 3
MAX_MELEE_MOBS: Final = 3
MAX_RANGED_MOBS: Final = 2
MAX_GROWING_PLANTS: Final = 10
MOB_DESPAWN_DISTANCE: Final = 14

LEVELS: Final = 9
"""Floors: overworld, dungeon, gnomish mines, sewers, vault, troll mines, fire realm, ice realm, graveyard."""
MONSTERS_KILLED_TO_CLEAR_LEVEL: Final = 8
"""Kills on a floor before its ladder down opens."""
LEVEL_ACHIEVEMENT: Final = (None, Achievement.ENTER_DUNGEON, Achievement.ENTER_GNOMISH_MINES, Achievement.ENTER_SEWERS,
                            Achievement.ENTER_VAULT, Achievement.ENTER_TROLL_MINES, Achievement.ENTER_FIRE_REALM,
                            Achievement.ENTER_ICE_REALM, Achievement.ENTER_GRAVEYARD)  # fmt: skip
FLOOR_SPECIES: Final = ((0, 0, 0), (2, 2, 2), (1, 1, 1), (2, 3, 3), (2, 4, 4), (1, 5, 5), (1, 6, 6), (1, 7, 7), (0, 0, 0))
"""Per floor, the (passive, melee, ranged) species that live there."""
FLOOR_HEALTH: Final = ((3.0, 5.0, 3.0), (4.0, 7.0, 5.0), (6.0, 9.0, 6.0), (8.0, 11.0, 8.0), (0.0, 12.0, 12.0),
                       (0.0, 20.0, 4.0), (0.0, 20.0, 14.0), (0.0, 24.0, 16.0), (0.0, 5.0, 3.0))  # fmt: skip
"""Per floor, fresh creature health (passive, melee, ranged); 0 where the floor has none."""
SPECIES_DAMAGE: Final = (
    ((2.0, 0.0, 0.0), (2.0, 0.0, 0.0)),
    ((4.0, 0.0, 0.0), (4.0, 0.0, 0.0)),
    ((3.0, 0.0, 0.0), (0.0, 3.0, 0.0)),
    ((5.0, 0.0, 0.0), (0.0, 0.0, 3.0)),
    ((6.0, 0.0, 0.0), (5.0, 0.0, 0.0)),
    ((6.0, 1.0, 1.0), (4.0, 3.0, 3.0)),
    ((3.0, 5.0, 0.0), (3.0, 5.0, 0.0)),
    ((4.0, 0.0, 5.0), (4.0, 0.0, 5.0)),
)
"""Per melee / ranged species, (melee hit, projectile) damage as (physical, fire, ice): the orc
mages throw fire, the kobolds ice, the deep things all three, and the elemental realms' creatures
add their realm's element."""
SPECIES_DEFENSE: Final = (
    (0.0, 0.0, 0.0),
    (0.0, 0.0, 0.0),
    (0.0, 0.0, 0.0),
    (0.0, 0.0, 0.0),
    (0.5, 0.0, 0.0),
    (0.2, 0.0, 0.0),
    (0.9, 1.0, 0.0),
    (0.9, 0.0, 1.0),
)
"""Per melee / ranged species, the fraction of (physical, fire, ice) damage it shrugs off: knights
and archers wear plate, the fire realm's creatures are immune to fire and the ice realm's to ice
(and both mostly to blades), so the elemental floors want the opposite element."""
ARMOUR_DEFENSE: Final = (0.1, 0.2)
"""Physical share blocked by one iron / diamond armour piece."""
ENCHANT_DEFENSE: Final = 0.2
"""Share of its element that one enchanted armour piece blocks."""
FLOOR_SPAWN: Final = ((0.1, 0.02, 0.05, 0.1),) + ((0.1, 0.06, 0.05, 0.0),) * 3 + ((0.0, 0.06, 0.05, 0.0),) * 5
"""Per floor, spawn probability for (passive, melee, ranged, melee at night)."""
PASSIVE_ACHIEVEMENT: Final = (Achievement.EAT_COW, Achievement.EAT_BAT, Achievement.EAT_SNAIL)
MELEE_ACHIEVEMENT: Final = (Achievement.DEFEAT_ZOMBIE, Achievement.DEFEAT_GNOME_WARRIOR, Achievement.DEFEAT_ORC_SOLIDER,
                            Achievement.DEFEAT_LIZARD, Achievement.DEFEAT_KNIGHT, Achievement.DEFEAT_TROLL,
                            Achievement.DEFEAT_PIGMAN, Achievement.DEFEAT_FROST_TROLL)  # fmt: skip
RANGED_ACHIEVEMENT: Final = (Achievement.DEFEAT_SKELETON, Achievement.DEFEAT_GNOME_ARCHER, Achievement.DEFEAT_ORC_MAGE,
                             Achievement.DEFEAT_KOBOLD, Achievement.DEFEAT_ARCHER, Achievement.DEFEAT_DEEP_THING,
                             Achievement.DEFEAT_FIRE_ELEMENTAL, Achievement.DEFEAT_ICE_ELEMENTAL)  # fmt: skip
LIT_FLOORS: Final = (True, False, False, False, False, False, True, True, True)
"""Floors lit throughout; on the others the player sees 3 tiles around itself and 4 around a torch."""

BOSS_EXTRA_DAMAGE: Final = 0.5
"""On the graveyard the player takes this much more damage."""
BOSS_WAVE_STEPS: Final = 7
"""After each wound the necromancer summons for this many steps before it can be struck again."""
SPELL_DAMAGE: Final = 6.0
"""Damage of a fireball or iceball at intelligence 1 (this build's figure)."""

PASSIVE_HEALTH: Final = 3.0
"""Health of the cows placed at world generation."""

_TIERS: Final = {
    3.0: (Achievement.MAKE_DIAMOND_SWORD, Achievement.MAKE_IRON_ARMOUR, Achievement.MAKE_DIAMOND_ARMOUR,
          Achievement.ENTER_GNOMISH_MINES, Achievement.ENTER_DUNGEON, Achievement.DEFEAT_GNOME_WARRIOR,
          Achievement.DEFEAT_GNOME_ARCHER, Achievement.DEFEAT_ORC_SOLIDER, Achievement.DEFEAT_ORC_MAGE,
          Achievement.EAT_BAT, Achievement.EAT_SNAIL, Achievement.FIND_BOW, Achievement.FIRE_BOW,
          Achievement.COLLECT_SAPPHIRE, Achievement.COLLECT_RUBY, Achievement.MAKE_DIAMOND_PICKAXE,
          Achievement.OPEN_CHEST, Achievement.DRINK_POTION),
    5.0: (Achievement.ENTER_SEWERS, Achievement.ENTER_VAULT, Achievement.ENTER_TROLL_MINES, Achievement.DEFEAT_LIZARD,
          Achievement.DEFEAT_KOBOLD, Achievement.DEFEAT_TROLL, Achievement.DEFEAT_DEEP_THING,
          Achievement.LEARN_FIREBALL, Achievement.CAST_FIREBALL, Achievement.LEARN_ICEBALL, Achievement.CAST_ICEBALL,
          Achievement.ENCHANT_SWORD, Achievement.ENCHANT_ARMOUR, Achievement.DEFEAT_KNIGHT, Achievement.DEFEAT_ARCHER),
    8.0: (Achievement.ENTER_FIRE_REALM, Achievement.ENTER_ICE_REALM, Achievement.ENTER_GRAVEYARD,
          Achievement.DEFEAT_PIGMAN, Achievement.DEFEAT_FIRE_ELEMENTAL, Achievement.DEFEAT_FROST_TROLL,
          Achievement.DEFEAT_ICE_ELEMENTAL, Achievement.DAMAGE_NECROMANCER, Achievement.DEFEAT_NECROMANCER),
}  # fmt: skip


def _rewards() -> torch.Tensor:
    r = torch.ones(NUM_ACHIEVEMENTS)
    for value, names in _TIERS.items():
        r[[int(a) for a in names]] = value
    return r


ACHIEVEMENT_REWARD: Final = _rewards()
REWARD_CEILING: Final = float(ACHIEVEMENT_REWARD.sum())
"""226: the score's normalizing denominator."""

SOLID: Final = torch.zeros(len(BlockType), dtype=torch.bool)
SOLID[[int(b) for b in (BlockType.STONE, BlockType.TREE, BlockType.COAL, BlockType.IRON, BlockType.DIAMOND,
                        BlockType.CRAFTING_TABLE, BlockType.FURNACE, BlockType.PLANT, BlockType.RIPE_PLANT,
                        BlockType.WALL, BlockType.WALL_MOSS, BlockType.STALAGMITE, BlockType.SAPPHIRE, BlockType.RUBY,
                        BlockType.CHEST, BlockType.FOUNTAIN, BlockType.FIRE_TREE, BlockType.ICE_SHRUB,
                        BlockType.GRAVE, BlockType.GRAVE2, BlockType.GRAVE3, BlockType.NECROMANCER,
                        BlockType.ENCHANTMENT_TABLE_FIRE, BlockType.ENCHANTMENT_TABLE_ICE)]] = True  # fmt: skip
"""Blocks that stop the player and creatures."""
WALKABLE: Final = torch.zeros(len(BlockType), dtype=torch.bool)
WALKABLE[[int(b) for b in (BlockType.GRASS, BlockType.SAND, BlockType.PATH, BlockType.FIRE_GRASS, BlockType.ICE_GRASS)]] = True
"""Blocks a creature (or the player) may step onto (water and lava stop creatures; lava kills the player)."""


_CACHE: dict[tuple, torch.Tensor] = {}


def device_table(key: object, device: torch.device, build: object) -> torch.Tensor:
    """A constant table on ``device``, copied there once (a per-step host copy would stall the stream)."""
    k = (key, device)
    t = _CACHE.get(k)
    if t is None:
        t = _CACHE[k] = torch.as_tensor(build() if callable(build) else build).to(device)
    return t
