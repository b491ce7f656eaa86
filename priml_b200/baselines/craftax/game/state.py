"""Batched state of the Craftax game (``priml/baselines/craftax/game/state.py``).

Every field is a tensor with the worker (environment) axis first, so one rollout
step is one batched tensor program on the device: no simulator process and no
host round trip. ``select`` merges two states row by row (auto-reset) and
``take`` gathers rows (dealing freshly generated worlds to finished workers).
"""

from __future__ import annotations

from dataclasses import dataclass, fields
from typing import Any

import torch
from torch import Tensor

from priml_b200.baselines.craftax.game import constants as C

__all__ = ["Creatures", "GameState", "empty_state"]


@dataclass(slots=True, kw_only=True)
class Creatures:
    """One class of creature: ``[envs, slots]`` records (``mask`` marks live slots)."""

    position: Tensor  # [E, S, 2] int64 (row, column)
    health: Tensor  # [E, S] float
    mask: Tensor  # [E, S] bool
    cooldown: Tensor  # [E, S] int32
    direction: Tensor  # [E, S, 2] int64 (projectiles only)

    @classmethod
    def empty(cls, envs: int, slots: int, device: torch.device) -> Creatures:
        return cls(position=torch.zeros(envs, slots, 2, dtype=torch.long, device=device),
                   health=torch.zeros(envs, slots, device=device),
                   mask=torch.zeros(envs, slots, dtype=torch.bool, device=device),
                   cooldown=torch.zeros(envs, slots, dtype=torch.int32, device=device),
                   direction=torch.zeros(envs, slots, 2, dtype=torch.long, device=device))  # fmt: skip


_COUNTS = ("wood", "stone", "coal", "iron", "diamond", "sapphire", "ruby", "sapling", "pickaxe", "sword", "arrows", "torches")


@dataclass(slots=True, kw_only=True)
class GameState:
    map: Tensor  # [E, H, W] int64 BlockType
    item_map: Tensor  # [E, H, W] int64 ItemType
    position: Tensor  # [E, 2] int64
    direction: Tensor  # [E] int64 Action of the last move (1..4)
    health: Tensor  # [E] float
    food: Tensor  # [E] int64
    drink: Tensor
    energy: Tensor
    hunger: Tensor  # [E] float accumulators
    thirst: Tensor
    fatigue: Tensor
    recover: Tensor
    sleeping: Tensor  # [E] bool
    wood: Tensor  # inventory counts [E] int64
    stone: Tensor
    coal: Tensor
    iron: Tensor
    diamond: Tensor
    sapphire: Tensor
    ruby: Tensor
    sapling: Tensor
    pickaxe: Tensor  # tool level 0..4 (none, wood, stone, iron, diamond)
    sword: Tensor
    arrows: Tensor
    torches: Tensor
    armour: Tensor  # [E, 4] int64: 0 none, 1 iron, 2 diamond
    passive: Creatures
    melee: Creatures
    ranged: Creatures
    projectiles: Creatures
    plant_position: Tensor  # [E, P, 2]
    plant_age: Tensor  # [E, P] int64
    plant_mask: Tensor  # [E, P] bool
    achievements: Tensor  # [E, 67] bool
    timestep: Tensor  # [E] int64
    light: Tensor  # [E] float daylight
    # floors: `map` / `item_map` hold the current floor; the others wait in the floor stores
    level: Tensor  # [E] int64
    floor_map: Tensor  # [E, L, H, W]
    floor_items: Tensor  # [E, L, H, W]
    ladder_down: Tensor  # [E, L, 2]
    ladder_up: Tensor  # [E, L, 2]
    kills: Tensor  # [E, L] monsters defeated per floor
    visited: Tensor  # [E, L] bool
    bow: Tensor  # [E]
    potions: Tensor  # [E, 6] red, green, blue, pink, cyan, yellow
    potion_effect: Tensor  # [E, 6] hidden effect of each colour (a permutation per world)
    xp: Tensor  # [E]
    dexterity: Tensor  # [E] attributes 1..5
    strength: Tensor
    intelligence: Tensor
    shots: Creatures  # the player's arrows and spells in flight (``cooldown`` holds the kind: 0 arrow, 1 fire, 2 ice)
    mana: Tensor  # [E]
    mana_regen: Tensor  # [E] float accumulator
    books: Tensor  # [E]
    spells: Tensor  # [E, 2] bool fireball, iceball learned
    sword_enchant: Tensor  # [E] 0 none, 1 fire, 2 ice
    bow_enchant: Tensor  # [E]
    armour_enchant: Tensor  # [E, 4]
    chests_opened: Tensor  # [E, L]
    resting: Tensor  # [E] bool
    boss_progress: Tensor  # [E] wounds dealt to the necromancer
    boss_wait: Tensor  # [E] steps until the necromancer can next be struck

    @property
    def num_envs(self) -> int:
        return int(self.timestep.shape[0])

    @property
    def device(self) -> torch.device:
        return self.timestep.device

    def _map(self, fn: Any, other: GameState) -> GameState:
        out: dict[str, Any] = {}
        for f in fields(self):
            a, b = getattr(self, f.name), getattr(other, f.name)
            if isinstance(a, Tensor):
                out[f.name] = fn(a, b)
            else:
                out[f.name] = Creatures(**{g.name: fn(getattr(a, g.name), getattr(b, g.name)) for g in fields(a)})
        return GameState(**out)

    def select(self, replace: Tensor, other: GameState) -> GameState:
        """Rows where ``replace`` is true come from ``other``."""
        return self._map(lambda a, b: torch.where(replace.view(-1, *([1] * (a.dim() - 1))), b, a), other)

    def take(self, rows: Tensor) -> GameState:
        return self._map(lambda a, b: a[rows], self)

    def state_dict(self) -> dict[str, Tensor]:
        out: dict[str, Tensor] = {}
        for f in fields(self):
            v = getattr(self, f.name)
            if isinstance(v, Tensor):
                out[f.name] = v.clone()  # the rules update some fields in place
            else:
                for g in fields(v):
                    out[f"{f.name}.{g.name}"] = getattr(v, g.name).clone()
        return out

    def load_state_dict(self, s: dict[str, Tensor]) -> None:
        for k, v in s.items():
            head, _, tail = k.partition(".")
            if tail:
                setattr(getattr(self, head), tail, v.clone())
            else:
                setattr(self, head, v.clone())


def empty_state(envs: int, device: torch.device) -> GameState:
    rows, cols = C.MAP_SIZE

    def z(dtype: torch.dtype = torch.long, *shape: int) -> Tensor:
        return torch.zeros(envs, *shape, dtype=dtype, device=device)

    counts = {name: z() for name in _COUNTS}
    return GameState(
        map=z(torch.long, rows, cols), item_map=z(torch.long, rows, cols), position=z(torch.long, 2),
        direction=torch.full((envs,), int(C.Action.DOWN), dtype=torch.long, device=device),
        health=torch.full((envs,), float(C.MAX_METER), device=device),
        food=torch.full((envs,), C.MAX_METER, dtype=torch.long, device=device),
        drink=torch.full((envs,), C.MAX_METER, dtype=torch.long, device=device),
        energy=torch.full((envs,), C.MAX_METER, dtype=torch.long, device=device),
        hunger=z(torch.float32), thirst=z(torch.float32), fatigue=z(torch.float32), recover=z(torch.float32),
        sleeping=z(torch.bool), armour=z(torch.long, 4),
        passive=Creatures.empty(envs, C.MAX_PASSIVE_MOBS, device),
        melee=Creatures.empty(envs, C.MAX_MELEE_MOBS, device),
        ranged=Creatures.empty(envs, C.MAX_RANGED_MOBS, device),
        projectiles=Creatures.empty(envs, 3, device),
        plant_position=z(torch.long, C.MAX_GROWING_PLANTS, 2), plant_age=z(torch.long, C.MAX_GROWING_PLANTS),
        plant_mask=z(torch.bool, C.MAX_GROWING_PLANTS), achievements=z(torch.bool, C.NUM_ACHIEVEMENTS),
        timestep=z(), light=torch.ones(envs, device=device),
        level=z(), floor_map=z(torch.long, C.LEVELS, rows, cols), floor_items=z(torch.long, C.LEVELS, rows, cols),
        ladder_down=z(torch.long, C.LEVELS, 2), ladder_up=z(torch.long, C.LEVELS, 2), kills=z(torch.long, C.LEVELS),
        visited=z(torch.bool, C.LEVELS), bow=z(), potions=z(torch.long, 6),
        potion_effect=torch.arange(6, device=device).expand(envs, 6).clone(), xp=z(),
        dexterity=torch.ones(envs, dtype=torch.long, device=device),
        strength=torch.ones(envs, dtype=torch.long, device=device),
        intelligence=torch.ones(envs, dtype=torch.long, device=device),
        shots=Creatures.empty(envs, 3, device),
        mana=torch.full((envs,), 9, dtype=torch.long, device=device), mana_regen=z(torch.float32), books=z(),
        spells=z(torch.bool, 2), sword_enchant=z(), bow_enchant=z(), armour_enchant=z(torch.long, 4),
        chests_opened=z(torch.long, C.LEVELS), resting=z(torch.bool), boss_progress=z(), boss_wait=z(), **counts,
    )  # fmt: skip
