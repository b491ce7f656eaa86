"""One batched step of the Craftax game on any of its nine floors (``priml/baselines/craftax/game/step.py``).

Order of operations per step (every rule is a masked tensor update over all
workers at once): sleeping workers act NOOP -> ladders (descend needs 8 kills on
the floor; creatures stay behind) -> crafting -> DO on the facing tile
(creatures first, then the block: mining, chests, water / fountain, plants) ->
placing -> potions, attribute level-ups, bow shots, spells, books and
enchanting -> movement -> creatures (move, attack, projectiles) -> the player's
arrows and spells -> spawning / despawning -> plants -> survival meters and mana
-> the necromancer's countdown -> achievements from the inventory -> reward.

The rules are Crafter's and Craftax's published ones for the overworld (tool
tiers for mining, crafting next to a table (and furnace), cows / zombies /
skeletons, food / drink / energy / recovery counters, sleeping, saplings that
ripen). Reward = newly unlocked achievements' rewards + 0.1 x the change in
health. An episode ends when health reaches 0, after 100,000 steps, or when the
necromancer on the graveyard has taken one wound per floor below the surface;
it can be struck only while none of its summons live and it is not summoning
(7 steps after each wound), and the graveyard hurts the player half again.
"""

from __future__ import annotations

import torch
from torch import Tensor

from priml_b200.baselines.craftax.game import constants as C
from priml_b200.baselines.craftax.game.constants import Achievement as A
from priml_b200.baselines.craftax.game.constants import Action as Act
from priml_b200.baselines.craftax.game.constants import BlockType as B
from priml_b200.baselines.craftax.game.constants import ItemType as I
from priml_b200.baselines.craftax.game.state import Creatures, GameState
from priml_b200.baselines.craftax.game.world import daylight

__all__ = ["is_done", "step"]

_DELTA = torch.zeros(len(Act), 2, dtype=torch.long)
_DELTA[Act.LEFT] = torch.tensor([0, -1])
_DELTA[Act.RIGHT] = torch.tensor([0, 1])
_DELTA[Act.UP] = torch.tensor([-1, 0])
_DELTA[Act.DOWN] = torch.tensor([1, 0])
_SWORD_DAMAGE = torch.tensor([1.0, 2.0, 3.0, 5.0, 8.0])
_PLANT_RIPE_AGE = 600
_GROUND = (B.GRASS, B.SAND, B.PATH, B.FIRE_GRASS, B.ICE_GRASS)
"""Tiles creatures walk on."""
_FLOOR_GROUND = (B.GRASS, B.PATH, B.PATH, B.PATH, B.PATH, B.PATH, B.FIRE_GRASS, B.ICE_GRASS, B.GRASS)
"""Per floor, the tile creatures spawn on."""
_CAP = C.MAX_METER


def _rows(s: GameState) -> Tensor:
    return torch.arange(s.num_envs, device=s.device)


def _in_bounds(pos: Tensor) -> Tensor:
    rows, cols = C.MAP_SIZE
    return (pos[..., 0] >= 0) & (pos[..., 0] < rows) & (pos[..., 1] >= 0) & (pos[..., 1] < cols)


_const = C.device_table


def _clamp(pos: Tensor) -> Tensor:
    rows, cols = C.MAP_SIZE
    return torch.stack([pos[..., 0].clamp(0, rows - 1), pos[..., 1].clamp(0, cols - 1)], -1)


def _tile(grid: Tensor, pos: Tensor) -> Tensor:
    """Block (or item) at ``pos`` [E, 2]; out-of-bounds positions read OUT_OF_BOUNDS."""
    p = _clamp(pos)
    v = grid[torch.arange(grid.shape[0], device=grid.device), p[:, 0], p[:, 1]]
    return torch.where(_in_bounds(pos), v, torch.full_like(v, int(B.OUT_OF_BOUNDS)))


def _set(grid: Tensor, pos: Tensor, value: Tensor | int, where: Tensor) -> Tensor:
    p = _clamp(pos)
    r = torch.arange(grid.shape[0], device=grid.device)
    old = grid[r, p[:, 0], p[:, 1]]
    new = value.expand_as(old).to(grid.dtype) if isinstance(value, Tensor) else torch.full_like(old, value)
    grid = grid.clone()
    grid[r, p[:, 0], p[:, 1]] = torch.where(where & _in_bounds(pos), new, old)
    return grid


def _occupied(s: GameState, pos: Tensor) -> Tensor:
    """``[E]`` true where a live creature (any class) stands at ``pos``."""
    hit = torch.zeros(s.num_envs, dtype=torch.bool, device=s.device)
    for mobs in (s.passive, s.melee, s.ranged):
        hit |= ((mobs.position == pos[:, None]).all(-1) & mobs.mask).any(-1)
    return hit


def _near(s: GameState, block: B, radius: int = 1) -> Tensor:
    """``[E]`` true where ``block`` lies in the (2 radius + 1)^2 window around the player (one gather)."""
    rows, cols = C.MAP_SIZE
    span = torch.arange(-radius, radius + 1, device=s.device)
    rr = (s.position[:, 0:1] + span)[:, :, None].expand(-1, -1, span.numel())
    cc = (s.position[:, 1:2] + span)[:, None, :].expand(-1, span.numel(), -1)
    inside = (rr >= 0) & (rr < rows) & (cc >= 0) & (cc < cols)
    e = torch.arange(s.num_envs, device=s.device)[:, None, None]
    window = s.map[e, rr.clamp(0, rows - 1), cc.clamp(0, cols - 1)]
    return ((window == int(block)) & inside).flatten(1).any(-1)


def _unlock(s: GameState, achievement: A, where: Tensor) -> None:
    s.achievements[:, int(achievement)] |= where


def _facing(s: GameState) -> Tensor:
    return s.position + _const("delta", s.device, _DELTA)[s.direction]


# ---------------------------------------------------------------- crafting
def _craft(s: GameState, a: Tensor) -> None:
    table = _near(s, B.CRAFTING_TABLE)
    furnace = _near(s, B.FURNACE)

    def make(act: Act, ok: Tensor, costs: dict[str, int]) -> Tensor:
        do = (a == int(act)) & ok
        for name, n in costs.items():
            do &= getattr(s, name) >= n
        for name, n in costs.items():
            setattr(s, name, getattr(s, name) - n * do.long())
        return do

    for act, level, costs, ok in (
        (Act.MAKE_WOOD_PICKAXE, 1, {"wood": 1}, table),
        (Act.MAKE_STONE_PICKAXE, 2, {"wood": 1, "stone": 1}, table),
        (Act.MAKE_IRON_PICKAXE, 3, {"wood": 1, "coal": 1, "iron": 1}, table & furnace),
        (Act.MAKE_DIAMOND_PICKAXE, 4, {"wood": 1, "diamond": 3}, table),
    ):
        s.pickaxe = torch.where(make(act, ok & (s.pickaxe < level), costs), level, s.pickaxe)
    for act, level, costs, ok in (
        (Act.MAKE_WOOD_SWORD, 1, {"wood": 1}, table),
        (Act.MAKE_STONE_SWORD, 2, {"wood": 1, "stone": 1}, table),
        (Act.MAKE_IRON_SWORD, 3, {"wood": 1, "coal": 1, "iron": 1}, table & furnace),
        (Act.MAKE_DIAMOND_SWORD, 4, {"wood": 1, "diamond": 2}, table),
    ):
        s.sword = torch.where(make(act, ok & (s.sword < level), costs), level, s.sword)
    s.arrows = torch.clamp(s.arrows + 2 * make(Act.MAKE_ARROW, table, {"wood": 1, "stone": 1}).long(), max=99)
    s.torches = torch.clamp(s.torches + 4 * make(Act.MAKE_TORCH, table, {"wood": 1, "coal": 1}).long(), max=99)
    for act, tier, costs, ach in ((Act.MAKE_IRON_ARMOUR, 1, {"iron": 3, "coal": 3}, A.MAKE_IRON_ARMOUR),
                                  (Act.MAKE_DIAMOND_ARMOUR, 2, {"diamond": 3}, A.MAKE_DIAMOND_ARMOUR)):  # fmt: skip
        slot_free = s.armour < tier
        do = make(act, table & furnace & slot_free.any(-1), costs)
        first = torch.argmax(slot_free.long(), dim=-1)
        upgraded = s.armour.clone()
        upgraded[_rows(s), first] = tier
        s.armour = torch.where(do[:, None], upgraded, s.armour)
        _unlock(s, ach, do)


# ---------------------------------------------------------------- DO
def _level_table(s: GameState, table: tuple, column: int) -> Tensor:
    return _const((id(table), column), s.device, lambda: [row[column] for row in table])[s.level]


def _species_damage(s: GameState, cls: int, column: int) -> Tensor:
    """(physical, fire, ice) damage ``[E, 3]`` dealt by the class-``cls`` species of the current floor
    (column 0 its melee hit, 1 its projectile)."""
    build = lambda: [C.SPECIES_DAMAGE[row[cls]][column] for row in C.FLOOR_SPECIES]  # noqa: E731
    return _const(("species_damage", cls, column), s.device, build)[s.level]


def _species_defense(s: GameState, cls: int) -> Tensor:
    """(physical, fire, ice) shares ``[E, 3]`` the class-``cls`` species of the current floor resists
    (passive creatures resist nothing)."""
    build = lambda: [C.SPECIES_DEFENSE[row[cls]] if cls > 0 else (0.0, 0.0, 0.0) for row in C.FLOOR_SPECIES]  # noqa: E731
    return _const(("species_defense", cls), s.device, build)[s.level]


def _in_element(amount: Tensor, element: Tensor) -> Tensor:
    """``[E, 3]`` damage vector with ``amount`` in slot ``element`` (0 physical, 1 fire, 2 ice)."""
    out = torch.zeros(*amount.shape, 3, device=amount.device, dtype=amount.dtype)
    return out.scatter(-1, element.long().unsqueeze(-1), amount.unsqueeze(-1))


def _player_damage(s: GameState) -> Tensor:
    """Sword damage ``[E, 3]`` (physical, fire, ice): the tier's figure as physical damage, strength
    adding a quarter per level above 1; an enchanted sword adds half the tier's figure in its element,
    intelligence adding a twentieth of that per level."""
    base = _const("sword", s.device, _SWORD_DAMAGE)[s.sword]
    physical = base * (1.0 + 0.25 * (s.strength - 1).float())
    element = 0.5 * base * (s.sword_enchant > 0).float() * (1.0 + 0.05 * (s.intelligence - 1).float())
    return _in_element(physical, torch.zeros_like(s.sword)) + _in_element(element, s.sword_enchant.clamp(min=0))


def _boss_vulnerable(s: GameState) -> Tensor:
    """The necromancer can be struck on the graveyard once its summons are dead and it has stopped summoning."""
    return (s.level == C.LEVELS - 1) & ~s.melee.mask.any(-1) & ~s.ranged.mask.any(-1) & (s.boss_wait <= 0)


def _wound_boss(s: GameState, striking: Tensor) -> None:
    hit = striking & _boss_vulnerable(s)
    s.boss_progress = s.boss_progress + hit.long()
    s.boss_wait = torch.where(hit, torch.full_like(s.boss_wait, C.BOSS_WAVE_STEPS), s.boss_wait)
    _unlock(s, A.DAMAGE_NECROMANCER, hit)


def _hit_creatures(s: GameState, target: Tensor, doing: Tensor, damage: Tensor) -> Tensor:
    """Damage the creature on ``target``; returns where a creature absorbed the blow."""
    absorbed = torch.zeros_like(doing)
    r = _rows(s)
    for cls, mobs in enumerate((s.passive, s.melee, s.ranged)):
        at = (mobs.position == target[:, None]).all(-1) & mobs.mask & doing[:, None] & ~absorbed[:, None]
        hit_any = at.any(-1)
        landed = ((1.0 - _species_defense(s, cls)) * damage).sum(-1)  # what gets through, summed over elements
        mobs.health = mobs.health - at.float() * landed[:, None]
        killed = at & (mobs.health <= 0)
        mobs.mask = mobs.mask & ~killed
        died = killed.any(-1)
        if cls == 0:  # eating the passive creature
            s.food = torch.where(died, torch.clamp(s.food + 6, max=_CAP), s.food)
            s.hunger = torch.where(died, torch.zeros_like(s.hunger), s.hunger)
        else:
            s.kills[r, s.level] = s.kills[r, s.level] + died.long()
        kinds = (C.PASSIVE_ACHIEVEMENT, C.MELEE_ACHIEVEMENT, C.RANGED_ACHIEVEMENT)[cls]
        ach = _const(("kill", cls), s.device, lambda: [int(kinds[row[cls]]) for row in C.FLOOR_SPECIES])[s.level]  # noqa: B023
        s.achievements[r, ach] |= died
        absorbed |= hit_any
    return absorbed


def _interact(s: GameState, a: Tensor, generator: torch.Generator | None) -> None:
    doing = a == int(Act.DO)
    target = _facing(s)
    doing = doing & ~_hit_creatures(s, target, doing, _player_damage(s))
    block = _tile(s.map, target)
    _wound_boss(s, doing & (block == int(B.NECROMANCER)))

    def mine(kind: B, tool: int, item: str) -> None:
        ok = doing & (block == int(kind)) & (s.pickaxe >= tool)
        setattr(s, item, torch.clamp(getattr(s, item) + ok.long(), max=_CAP))
        s.map = _set(s.map, target, int(B.PATH), ok)

    wood = doing & (block == int(B.TREE))
    s.wood = torch.clamp(s.wood + wood.long(), max=_CAP)
    mine(B.STONE, 1, "stone")
    mine(B.COAL, 1, "coal")
    mine(B.IRON, 2, "iron")
    mine(B.DIAMOND, 3, "diamond")
    mine(B.SAPPHIRE, 4, "sapphire")
    mine(B.RUBY, 4, "ruby")
    sapling = doing & (block == int(B.GRASS)) & (torch.rand(s.num_envs, device=s.device, generator=generator) < 0.1)
    s.sapling = torch.clamp(s.sapling + sapling.long(), max=_CAP)
    chest = doing & (block == int(B.CHEST))
    _open_chest(s, chest, generator)
    s.map = _set(s.map, target, int(B.PATH), chest)
    drink = doing & ((block == int(B.WATER)) | (block == int(B.FOUNTAIN)))
    s.drink = torch.where(drink, torch.clamp(s.drink + 1, max=_CAP), s.drink)
    s.thirst = torch.where(drink, torch.zeros_like(s.thirst), s.thirst)
    _unlock(s, A.COLLECT_DRINK, drink)
    eat = doing & (block == int(B.RIPE_PLANT))
    s.food = torch.where(eat, torch.clamp(s.food + 4, max=_CAP), s.food)
    s.hunger = torch.where(eat, torch.zeros_like(s.hunger), s.hunger)
    s.map = _set(s.map, target, int(B.PLANT), eat)
    at_plant = (s.plant_position == target[:, None]).all(-1) & s.plant_mask & eat[:, None]
    s.plant_age = torch.where(at_plant, torch.zeros_like(s.plant_age), s.plant_age)
    _unlock(s, A.EAT_PLANT, eat)


def _open_chest(s: GameState, opening: Tensor, generator: torch.Generator | None) -> None:
    """Loot (this build's table): 1-4 arrows, and each with probability 1/2: 1-2 torches, a potion
    of a random colour, 1 iron; 1 diamond with probability 1/10. The first chest on a floor below
    the surface also holds a bow if the player has none, and the first on the sewers and on the
    vault a spellbook."""
    dev, n = s.device, s.num_envs

    def roll(p: float) -> Tensor:
        return opening & (torch.rand(n, device=dev, generator=generator) < p)

    s.arrows = torch.clamp(s.arrows + opening.long() * torch.randint(1, 5, (n,), device=dev, generator=generator), max=99)
    s.torches = torch.clamp(s.torches + roll(0.5).long() * torch.randint(1, 3, (n,), device=dev, generator=generator), max=99)
    colour = torch.randint(0, 6, (n,), device=dev, generator=generator)
    got = roll(0.5)
    s.potions[_rows(s), colour] = s.potions[_rows(s), colour] + got.long()
    s.iron = torch.clamp(s.iron + roll(0.5).long(), max=_CAP)
    s.diamond = torch.clamp(s.diamond + roll(0.1).long(), max=_CAP)
    bow = opening & (s.bow == 0) & (s.level > 0)
    s.bow = s.bow + bow.long()
    first_here = opening & (s.chests_opened[_rows(s), s.level] == 0)
    s.books = s.books + (first_here & ((s.level == 3) | (s.level == 4))).long()  # a spellbook in each
    s.chests_opened[_rows(s), s.level] += opening.long()
    _unlock(s, A.OPEN_CHEST, opening)
    _unlock(s, A.FIND_BOW, bow)


_POTION_ACTIONS = (Act.DRINK_POTION_RED, Act.DRINK_POTION_GREEN, Act.DRINK_POTION_BLUE, Act.DRINK_POTION_PINK,
                   Act.DRINK_POTION_CYAN, Act.DRINK_POTION_YELLOW)  # fmt: skip


def _abilities(s: GameState, a: Tensor) -> None:
    r = _rows(s)
    for colour, act in enumerate(_POTION_ACTIONS):
        drink = (a == int(act)) & (s.potions[:, colour] >= 1)
        s.potions[:, colour] = s.potions[:, colour] - drink.long()
        effect = s.potion_effect[:, colour]
        # this build's effects: heal 8 / hurt 3 / energy +8 / energy -3 / drink +8 / drink -3
        s.health = torch.where(drink & (effect == 0), s.health + 8, torch.where(drink & (effect == 1), s.health - 3, s.health))
        s.energy = torch.where(drink & (effect == 2), s.energy + 8, torch.where(drink & (effect == 3), s.energy - 3, s.energy))
        s.drink = torch.where(drink & (effect == 4), s.drink + 8, torch.where(drink & (effect == 5), s.drink - 3, s.drink))
        _unlock(s, A.DRINK_POTION, drink)
    for act, name in ((Act.LEVEL_UP_DEXTERITY, "dexterity"), (Act.LEVEL_UP_STRENGTH, "strength"),
                      (Act.LEVEL_UP_INTELLIGENCE, "intelligence")):  # fmt: skip
        up = (a == int(act)) & (s.xp >= 1) & (getattr(s, name) < 5)
        setattr(s, name, getattr(s, name) + up.long())
        s.xp = s.xp - up.long()
    # a bow shot or a spell leaves the player's tile and flies one tile per step
    room = ~s.shots.mask.all(-1)
    shoot = (a == int(Act.SHOOT_ARROW)) & (s.bow >= 1) & (s.arrows >= 1) & room
    fire = (a == int(Act.CAST_FIREBALL)) & s.spells[:, 0] & (s.mana >= 2) & room
    ice = (a == int(Act.CAST_ICEBALL)) & s.spells[:, 1] & (s.mana >= 2) & room
    _launch(s, shoot | fire | ice, fire.int() + 2 * ice.int())
    s.arrows = s.arrows - shoot.long()
    s.mana = s.mana - 2 * (fire | ice).long()
    _unlock(s, A.FIRE_BOW, shoot)
    _unlock(s, A.CAST_FIREBALL, fire)
    _unlock(s, A.CAST_ICEBALL, ice)
    # a book teaches a spell not yet known (fireball first), and is spent either way
    reading = (a == int(Act.READ_BOOK)) & (s.books >= 1)
    learn = torch.where(~s.spells[:, 0], 0, torch.where(~s.spells[:, 1], 1, 0))
    s.spells[r, learn] |= reading
    s.books = s.books - reading.long()
    _unlock(s, A.LEARN_FIREBALL, reading & (learn == 0))
    _unlock(s, A.LEARN_ICEBALL, reading & (learn == 1))
    _enchant(s, a)


def _launch(s: GameState, firing: Tensor, kind: Tensor) -> None:
    r = _rows(s)
    first = torch.argmax((~s.shots.mask).long(), -1)
    d = _const("delta", s.device, _DELTA)[s.direction]
    sh = s.shots
    pos, dirn, mask, kinds = sh.position.clone(), sh.direction.clone(), sh.mask.clone(), sh.cooldown.clone()
    pos[r, first] = torch.where(firing[:, None], s.position, pos[r, first])
    dirn[r, first] = torch.where(firing[:, None], d, dirn[r, first])
    mask[r, first] = mask[r, first] | firing
    kinds[r, first] = torch.where(firing, kind.to(kinds.dtype), kinds[r, first])
    sh.position, sh.direction, sh.mask, sh.cooldown = pos, dirn, mask, kinds


def _enchant(s: GameState, a: Tensor) -> None:
    """At an enchantment table, 9 mana and a gem (ruby at a fire table, sapphire at an ice one) bind
    the table's element to the sword, the bow, or the first armour piece that is bare or holds the
    other element."""
    fire_table, ice_table = _near(s, B.ENCHANTMENT_TABLE_FIRE), _near(s, B.ENCHANTMENT_TABLE_ICE)
    element = torch.where(fire_table, 1, 2)
    gem = torch.where(fire_table, s.ruby, s.sapphire)
    ready = (fire_table | ice_table) & (s.mana >= 9) & (gem >= 1)
    sword = ready & (a == int(Act.ENCHANT_SWORD)) & (s.sword >= 1)
    bow = ready & (a == int(Act.ENCHANT_BOW)) & (s.bow >= 1)
    fits = (s.armour > 0) & (s.armour_enchant != element[:, None])
    armour = ready & (a == int(Act.ENCHANT_ARMOUR)) & fits.any(-1)
    s.sword_enchant = torch.where(sword, element, s.sword_enchant)
    s.bow_enchant = torch.where(bow, element, s.bow_enchant)
    piece = torch.argmax((fits & (s.armour_enchant == 0)).long() * 2 + fits.long(), -1)
    r = _rows(s)
    s.armour_enchant[r, piece] = torch.where(armour, element, s.armour_enchant[r, piece])
    done = sword | bow | armour
    s.ruby = s.ruby - (done & (element == 1)).long()
    s.sapphire = s.sapphire - (done & (element == 2)).long()
    s.mana = s.mana - 9 * done.long()
    _unlock(s, A.ENCHANT_SWORD, sword)
    _unlock(s, A.ENCHANT_ARMOUR, armour)


def _fly_shots(s: GameState) -> None:
    shots = s.shots
    shots.position = shots.position + shots.direction * shots.mask[..., None].long()
    # arrows: 2, dexterity adding a quarter per level, an enchanted bow half again; spells: intelligence
    # adding a tenth per level
    # physical, an enchanted bow adding half again in its element
    arrow_hit = 2.0 * (1.0 + 0.25 * (s.dexterity - 1).float())
    arrow = _in_element(arrow_hit, torch.zeros_like(s.bow_enchant))
    arrow = arrow + _in_element(0.5 * arrow_hit * (s.bow_enchant > 0).float(), s.bow_enchant.clamp(min=0))
    spell = C.SPELL_DAMAGE * (1.0 + 0.1 * (s.intelligence - 1).float())
    for slot in range(shots.mask.shape[1]):
        live = shots.mask[:, slot]
        kind = shots.cooldown[:, slot]  # 0 arrow, 1 fireball, 2 iceball: the spell's element is its kind
        damage = torch.where((kind == 0)[:, None], arrow, _in_element(spell, kind.clamp(0, 2)))
        hit = _hit_creatures(s, shots.position[:, slot], live, damage)
        b = _tile(s.map, shots.position[:, slot])
        passable = torch.stack([b == int(g) for g in (*_GROUND, B.WATER, B.LAVA)]).any(0)
        shots.mask[:, slot] = live & ~hit & passable


def _change_floor(s: GameState, a: Tensor) -> None:
    here = _tile(s.item_map, s.position)
    r, lvl = _rows(s), s.level
    cleared = s.kills[r, lvl] >= C.MONSTERS_KILLED_TO_CLEAR_LEVEL
    down = (a == int(Act.DESCEND)) & (here == int(I.LADDER_DOWN)) & cleared & (lvl < C.LEVELS - 1)
    up = (a == int(Act.ASCEND)) & (here == int(I.LADDER_UP)) & (lvl > 0)
    move = down | up
    if s.device.type == "cpu" and not bool(move.any()):  # on the GPU a host read costs more than the swap
        return
    s.floor_map[r, lvl] = torch.where(move[:, None, None], s.map, s.floor_map[r, lvl])
    s.floor_items[r, lvl] = torch.where(move[:, None, None], s.item_map, s.floor_items[r, lvl])
    new = lvl + down.long() - up.long()
    s.map = torch.where(move[:, None, None], s.floor_map[r, new], s.map)
    s.item_map = torch.where(move[:, None, None], s.floor_items[r, new], s.item_map)
    s.position = torch.where(down[:, None], s.ladder_up[r, new], torch.where(up[:, None], s.ladder_down[r, new], s.position))
    s.level = new
    for mobs in (s.passive, s.melee, s.ranged, s.projectiles, s.shots):  # creatures stay behind (and despawn)
        mobs.mask = mobs.mask & ~move[:, None]
    first = move & ~s.visited[r, new]
    s.visited[r, new] |= move
    s.xp = s.xp + first.long()
    for level, ach in enumerate(C.LEVEL_ACHIEVEMENT):
        if ach is not None:
            _unlock(s, ach, move & (new == level))


# ---------------------------------------------------------------- placing
def _place(s: GameState, a: Tensor) -> None:
    target = _facing(s)
    block = _tile(s.map, target)
    free = ~_occupied(s, target) & _in_bounds(target)
    ground = (block == int(B.GRASS)) | (block == int(B.SAND)) | (block == int(B.PATH))

    stone = (a == int(Act.PLACE_STONE)) & (s.stone >= 1) & free & (ground | (block == int(B.WATER)) | (block == int(B.LAVA)))
    s.map = _set(s.map, target, int(B.STONE), stone)
    s.stone = s.stone - stone.long()
    _unlock(s, A.PLACE_STONE, stone)
    table = (a == int(Act.PLACE_TABLE)) & (s.wood >= 1) & free & ground
    s.map = _set(s.map, target, int(B.CRAFTING_TABLE), table)
    s.wood = s.wood - table.long()
    _unlock(s, A.PLACE_TABLE, table)
    furnace = (a == int(Act.PLACE_FURNACE)) & (s.stone >= 1) & free & ground & _near(s, B.CRAFTING_TABLE)
    s.map = _set(s.map, target, int(B.FURNACE), furnace)
    s.stone = s.stone - furnace.long()
    _unlock(s, A.PLACE_FURNACE, furnace)
    slot_free = ~s.plant_mask
    plant = (a == int(Act.PLACE_PLANT)) & (s.sapling >= 1) & free & (block == int(B.GRASS)) & slot_free.any(-1)
    s.map = _set(s.map, target, int(B.PLANT), plant)
    s.sapling = s.sapling - plant.long()
    first = torch.argmax(slot_free.long(), dim=-1)
    r = _rows(s)
    pos, age, mask = s.plant_position.clone(), s.plant_age.clone(), s.plant_mask.clone()
    pos[r, first] = torch.where(plant[:, None], target, pos[r, first])
    age[r, first] = torch.where(plant, torch.zeros_like(age[r, first]), age[r, first])
    mask[r, first] = mask[r, first] | plant
    s.plant_position, s.plant_age, s.plant_mask = pos, age, mask
    _unlock(s, A.PLACE_PLANT, plant)
    torch_ok = (a == int(Act.PLACE_TORCH)) & (s.torches >= 1) & ground & (_tile(s.item_map, target) == int(I.NONE))
    s.item_map = _set(s.item_map, target, int(I.TORCH), torch_ok)
    s.torches = s.torches - torch_ok.long()
    _unlock(s, A.PLACE_TORCH, torch_ok)


# ---------------------------------------------------------------- movement
def _move(s: GameState, a: Tensor) -> None:
    moving = (a >= int(Act.LEFT)) & (a <= int(Act.DOWN))
    s.direction = torch.where(moving, a, s.direction)
    target = s.position + _const("delta", s.device, _DELTA)[a]
    block = _tile(s.map, target)
    ok = moving & _in_bounds(target) & ~_occupied(s, target)
    ok &= (block == int(B.GRASS)) | (block == int(B.SAND)) | (block == int(B.PATH)) | (block == int(B.LAVA))
    s.position = torch.where(ok[:, None], target, s.position)
    s.health = torch.where(_tile(s.map, s.position) == int(B.LAVA), torch.zeros_like(s.health), s.health)


# ---------------------------------------------------------------- creatures
def _random_step(mobs: Creatures, generator: torch.Generator | None) -> Tensor:
    e, k = mobs.mask.shape
    choice = torch.randint(0, 5, (e, k), device=mobs.mask.device, generator=generator)  # 0 = stay
    return _DELTA.to(mobs.mask.device)[choice]


def _try_move(s: GameState, mobs: Creatures, step: Tensor, allowed: tuple[B, ...],
              also: tuple[B, Tensor] | None = None) -> None:  # fmt: skip
    """Move each creature by ``step`` onto a free ``allowed`` tile (or ``also[0]`` where ``also[1]``)."""
    for slot in range(mobs.mask.shape[1]):
        pos = mobs.position[:, slot]
        target = pos + step[:, slot]
        block = _tile(s.map, target)
        ok = mobs.mask[:, slot] & _in_bounds(target) & ~_occupied(s, target) & ~(target == s.position).all(-1)
        fits = torch.stack([block == int(b) for b in allowed]).any(0)
        if also is not None:
            fits |= (block == int(also[0])) & also[1]
        ok &= fits
        mobs.position[:, slot] = torch.where(ok[:, None], target, pos)


def _damage_to_player(s: GameState, damage: Tensor) -> Tensor:
    """What a ``[E, 3]`` (physical, fire, ice) blow takes from the player: each iron piece blocks a
    tenth and each diamond piece a fifth of the physical part, each piece enchanted in an element a
    fifth of that element; the graveyard adds half again."""
    worn = s.armour > 0
    physical = C.ARMOUR_DEFENSE[0] * (s.armour == 1).sum(-1).float() + C.ARMOUR_DEFENSE[1] * (s.armour == 2).sum(-1).float()
    fire = C.ENCHANT_DEFENSE * (worn & (s.armour_enchant == 1)).sum(-1).float()
    ice = C.ENCHANT_DEFENSE * (worn & (s.armour_enchant == 2)).sum(-1).float()
    resisted = torch.stack([physical, fire, ice], -1).clamp(max=1.0)
    boss = 1.0 + C.BOSS_EXTRA_DAMAGE * (s.level == C.LEVELS - 1).float()
    return ((1.0 - resisted) * damage).sum(-1) * boss


def _creatures(s: GameState, generator: torch.Generator | None) -> None:
    dev = s.device
    # cows wander
    _try_move(s, s.passive, _random_step(s.passive, generator), _GROUND)
    # zombies chase when close, else wander; adjacent ones attack every 5 steps
    offset = s.position[:, None] - s.melee.position
    dist = offset.abs().sum(-1)
    toward = torch.where((offset[..., 0].abs() >= offset[..., 1].abs())[..., None],
                         torch.stack([offset[..., 0].sign(), torch.zeros_like(offset[..., 0])], -1),
                         torch.stack([torch.zeros_like(offset[..., 1]), offset[..., 1].sign()], -1))  # fmt: skip
    chase = (dist < 8) & (torch.rand(dist.shape, device=dev, generator=generator) < 0.8)
    step = torch.where(chase[..., None], toward, _random_step(s.melee, generator))
    _try_move(s, s.melee, step, _GROUND)
    dist = (s.position[:, None] - s.melee.position).abs().sum(-1)
    attack = s.melee.mask & (dist <= 1) & (s.melee.cooldown <= 0)
    melee_hit = _species_damage(s, 1, 0)
    asleep = _in_element(torch.full_like(s.health, 7.0), torch.zeros_like(s.level))  # a sleeper takes a heavy blow
    damage = torch.where(s.sleeping[:, None], asleep, melee_hit)
    s.health = s.health - attack.sum(-1).float() * _damage_to_player(s, damage)
    s.melee.cooldown = torch.where(attack, torch.full_like(s.melee.cooldown, 5), (s.melee.cooldown - 1).clamp(min=0))
    # skeletons keep to the caves and shoot along rows / columns when the player is within 4 tiles
    _try_move(s, s.ranged, _random_step(s.ranged, generator), _GROUND[2:], also=(B.GRASS, s.level > 0))
    offset = s.position[:, None] - s.ranged.position
    aligned = (offset == 0).any(-1) & (offset.abs().sum(-1) <= 4)
    shoot = s.ranged.mask & aligned & (s.ranged.cooldown <= 0)
    s.ranged.cooldown = torch.where(shoot, torch.full_like(s.ranged.cooldown, 4), (s.ranged.cooldown - 1).clamp(min=0))
    proj = s.projectiles
    for slot in range(s.ranged.mask.shape[1]):
        want = shoot[:, slot]
        free = ~proj.mask
        first = torch.argmax(free.long(), -1)
        put = want & free.any(-1)
        r = _rows(s)
        d = offset[:, slot].sign()
        pos, dirn, mask = proj.position.clone(), proj.direction.clone(), proj.mask.clone()
        pos[r, first] = torch.where(put[:, None], s.ranged.position[:, slot], pos[r, first])
        dirn[r, first] = torch.where(put[:, None], d, dirn[r, first])
        mask[r, first] = mask[r, first] | put
        proj.position, proj.direction, proj.mask = pos, dirn, mask
    # arrows fly one tile per step: they hurt the player they reach and stop at solid tiles
    proj.position = proj.position + proj.direction * proj.mask[..., None].long()
    hit = proj.mask & (proj.position == s.position[:, None]).all(-1)
    s.health = s.health - hit.sum(-1).float() * _damage_to_player(s, _species_damage(s, 2, 1))
    blocked = torch.zeros_like(proj.mask)
    for slot in range(proj.mask.shape[1]):
        b = _tile(s.map, proj.position[:, slot])
        blocked[:, slot] = ~(torch.stack([b == int(g) for g in (*_GROUND, B.WATER, B.LAVA)]).any(0))
    proj.mask = proj.mask & ~hit & ~blocked


def _spawn(s: GameState, generator: torch.Generator | None) -> None:
    dev, e = s.device, s.num_envs
    rows, cols = C.MAP_SIZE
    night = s.light < 0.5
    surface = s.level == 0
    melee_chance = torch.where(night & surface, _level_table(s, C.FLOOR_SPAWN, 3), _level_table(s, C.FLOOR_SPAWN, 1))
    grass_or_path = _const("ground", dev, lambda: [int(b) for b in _FLOOR_GROUND])[s.level]
    ranged_tile = torch.where(surface, int(B.PATH), grass_or_path)  # overworld skeletons keep to tunnels
    # the graveyard's creatures are the necromancer's summons: they come only while it summons
    summoning = (s.level != C.LEVELS - 1) | (s.boss_wait > 0)
    for cls, mobs, chance, tile, min_dist in (
        (0, s.passive, _level_table(s, C.FLOOR_SPAWN, 0), grass_or_path, 3),
        (1, s.melee, melee_chance * summoning, grass_or_path, 6),
        (2, s.ranged, _level_table(s, C.FLOOR_SPAWN, 2) * summoning, ranged_tile, 4),
    ):  # fmt: skip
        far = (mobs.position - s.position[:, None]).abs().max(-1).values > C.MOB_DESPAWN_DISTANCE
        mobs.mask = mobs.mask & ~far
        pos = torch.stack([(s.position[:, 0] + torch.randint(-9, 10, (e,), device=dev, generator=generator)).clamp(0, rows - 1),
                           (s.position[:, 1] + torch.randint(-9, 10, (e,), device=dev, generator=generator)).clamp(0, cols - 1)], -1)  # fmt: skip
        ok = torch.rand(e, device=dev, generator=generator) < chance
        ok &= (_tile(s.map, pos) == tile) & ~_occupied(s, pos) & ~(pos == s.position).all(-1)
        ok &= (pos - s.position).abs().sum(-1) >= min_dist
        free = ~mobs.mask
        ok &= free.any(-1)
        first = torch.argmax(free.long(), -1)
        r = _rows(s)
        health = _level_table(s, C.FLOOR_HEALTH, cls)
        p, h, m, cd = mobs.position.clone(), mobs.health.clone(), mobs.mask.clone(), mobs.cooldown.clone()
        p[r, first] = torch.where(ok[:, None], pos, p[r, first])
        h[r, first] = torch.where(ok, health, h[r, first])
        m[r, first] = m[r, first] | ok
        cd[r, first] = torch.where(ok, torch.zeros_like(cd[r, first]), cd[r, first])
        mobs.position, mobs.health, mobs.mask, mobs.cooldown = p, h, m, cd


def _plants(s: GameState) -> None:
    """Saplings grow on the surface; they wait (not ageing) while the player is below."""
    surface = s.level == 0
    s.plant_age = s.plant_age + (s.plant_mask & surface[:, None]).long()
    for slot in range(s.plant_mask.shape[1]):
        pos = s.plant_position[:, slot]
        here = _tile(s.map, pos)
        live = s.plant_mask[:, slot] & (~surface | (here == int(B.PLANT)) | (here == int(B.RIPE_PLANT)))
        s.plant_mask[:, slot] = live  # a plant removed stops growing
        ripe = live & surface & (s.plant_age[:, slot] >= _PLANT_RIPE_AGE) & (here == int(B.PLANT))
        s.map = _set(s.map, pos, int(B.RIPE_PLANT), ripe)


# ---------------------------------------------------------------- survival
def _survive(s: GameState, a: Tensor) -> None:
    # mana: one point per 20 steps (10 asleep), intelligence adding a quarter per level; cap 6 + 3 x intelligence
    s.mana_regen = s.mana_regen + torch.where(s.sleeping, 0.1, 0.05) * (1.0 + 0.25 * (s.intelligence - 1).float())
    s.mana = torch.minimum(torch.where(s.mana_regen >= 1, s.mana + 1, s.mana).clamp(min=0), 6 + 3 * s.intelligence)
    s.mana_regen = torch.where(s.mana_regen >= 1, s.mana_regen - 1, s.mana_regen)
    s.resting = a == int(Act.REST)
    start = (a == int(Act.SLEEP)) & (s.energy < _CAP)
    s.sleeping = s.sleeping | start
    slow = torch.where(s.sleeping, 0.5, 1.0)
    s.hunger = s.hunger + slow
    s.food = torch.where(s.hunger > 25, s.food - 1, s.food)
    s.hunger = torch.where(s.hunger > 25, torch.zeros_like(s.hunger), s.hunger)
    s.thirst = s.thirst + slow
    s.drink = torch.where(s.thirst > 20, s.drink - 1, s.drink)
    s.thirst = torch.where(s.thirst > 20, torch.zeros_like(s.thirst), s.thirst)
    s.fatigue = torch.where(s.sleeping, torch.clamp(s.fatigue - 1, max=0.0), s.fatigue + 1)
    s.energy = torch.where(s.fatigue > 30, s.energy - 1, s.energy)
    s.energy = torch.where(s.fatigue < -10, s.energy + 1, s.energy)
    s.fatigue = torch.where((s.fatigue > 30) | (s.fatigue < -10), torch.zeros_like(s.fatigue), s.fatigue)
    fine = (s.food > 0) & (s.drink > 0) & ((s.energy > 0) | s.sleeping)
    s.recover = s.recover + torch.where(fine, torch.where(s.sleeping | s.resting, 2.0, 1.0), torch.where(s.sleeping, -0.5, -1.0))
    s.health = torch.where(s.recover > 25, s.health + 1, s.health)
    s.health = torch.where(s.recover < -15, s.health - 1, s.health)
    s.recover = torch.where((s.recover > 25) | (s.recover < -15), torch.zeros_like(s.recover), s.recover)
    woke = s.sleeping & (s.energy >= _CAP)
    s.sleeping = s.sleeping & ~woke
    _unlock(s, A.WAKE_UP, woke)
    s.food, s.drink, s.energy = (x.clamp(0, _CAP) for x in (s.food, s.drink, s.energy))  # potions may overshoot
    s.health = s.health.clamp(max=float(_CAP))


_THRESHOLDS = (("wood", 1, A.COLLECT_WOOD), ("stone", 1, A.COLLECT_STONE), ("coal", 1, A.COLLECT_COAL),
               ("iron", 1, A.COLLECT_IRON), ("diamond", 1, A.COLLECT_DIAMOND), ("sapling", 1, A.COLLECT_SAPLING),
               ("sapphire", 1, A.COLLECT_SAPPHIRE), ("ruby", 1, A.COLLECT_RUBY),
               ("arrows", 1, A.MAKE_ARROW), ("torches", 1, A.MAKE_TORCH), ("pickaxe", 1, A.MAKE_WOOD_PICKAXE),
               ("pickaxe", 2, A.MAKE_STONE_PICKAXE), ("pickaxe", 3, A.MAKE_IRON_PICKAXE),
               ("pickaxe", 4, A.MAKE_DIAMOND_PICKAXE), ("sword", 1, A.MAKE_WOOD_SWORD), ("sword", 2, A.MAKE_STONE_SWORD),
               ("sword", 3, A.MAKE_IRON_SWORD), ("sword", 4, A.MAKE_DIAMOND_SWORD))  # fmt: skip


def step(s: GameState, action: Tensor, *, generator: torch.Generator | None = None) -> tuple[GameState, Tensor]:
    """Advance every worker by one step; returns the state (updated in place) and the reward ``[E]``."""
    before = s.achievements.clone()
    health_before = s.health.clone()
    a = torch.where(s.sleeping, torch.full_like(action, int(Act.NOOP)), action.long())
    _change_floor(s, a)
    _craft(s, a)
    _interact(s, a, generator)
    _place(s, a)
    _abilities(s, a)
    _move(s, a)
    _creatures(s, generator)
    _fly_shots(s)
    _spawn(s, generator)
    _plants(s)
    _survive(s, a)
    s.boss_wait = (s.boss_wait - (s.level == C.LEVELS - 1).long()).clamp(min=0)
    _unlock(s, A.DEFEAT_NECROMANCER, s.boss_progress >= C.LEVELS - 1)
    for name, n, ach in _THRESHOLDS:
        _unlock(s, ach, getattr(s, name) >= n)
    newly = (s.achievements & ~before).float()
    reward = (newly * _const("reward", s.device, C.ACHIEVEMENT_REWARD)).sum(-1) + 0.1 * (s.health - health_before)
    s.timestep = s.timestep + 1
    s.light = daylight(s.timestep)
    return s, reward


def is_done(s: GameState) -> Tensor:
    """Death, the time limit, or the necromancer's defeat (after one wound per floor below the surface)."""
    return (s.health <= 0) | (s.timestep >= C.MAX_TIMESTEPS) | (s.boss_progress >= C.LEVELS - 1)
